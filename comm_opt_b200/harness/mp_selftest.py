"""Multi-GPU self-test of the fused collective and the TP decode runner (one process per GPU).

    timeout -k 60 600 python -m torch.distributed.run --standalone --nproc-per-node 2 \
        -m comm_opt_b200.harness.mp_selftest --parts functional,decode
    NCCL_NVLS_ENABLE=0 timeout -k 60 300 python -m torch.distributed.run --standalone --nproc-per-node 2 \
        -m comm_opt_b200.harness.mp_selftest --parts fault

Parts:
  functional - every variant (NVLS ones when the heap has a multicast object) x dtypes x shapes
               against an fp32 NCCL all-reduce oracle (relative error <= 2^-5, the reference's
               criterion), bitwise-identical results on every rank, plain all-reduce, small all-gather,
               the interleaving test (exp/M16_epoch_fix/test_interleave.py) in eager and graph mode,
               and a late rank (one rank sleeps before launching).
  fault      - fault injection on the host: one rank skips a call, the others' bounded waits run out,
               they report TPCommTimeout, every rank calls reset() and the next calls are correct.
               Uses the CUDA-IPC heap (never bound to a multicast object) and plain peer loads.
  leave      - a rank leaves between steps (nothing in flight) and posts it in the store; the others stop
               before their next launch (RankMonitor.sync), no bounded wait runs out. Use the CUDA-IPC
               heap's environment (NCCL_NVLS_ENABLE=0), as for `fault`.
  stress     - fused calls and layer boundaries checked call by call while a side stream runs large
               GEMMs on every SM (memory-ordering stress under concurrent compute).
  decode     - tiny Llama-shaped model at TP = world vs the unsharded fp32 forward (logits), and
               identical greedy tokens on every rank.
  decode_fused - the same with the layer boundaries fused (GEMM push epilogue -> all-reduce + RMSNorm
               inside the next GEMM); decode_fused_epi also moves SiLU * up and RoPE + KV append
               into the consumer GEMMs' epilogues; decode_nccl runs the baseline step (NCCL all-reduce +
               add/RMSNorm kernel) through the same runner, decode_vllm the reference's baseline stack (vLLM
               custom all-reduce + vLLM fused_add_rms_norm); decode_qkv_bias runs the fused step on the
               Qwen2.5 attention shape (QKV bias, 5 query heads per KV head at 4 ranks); decode_mixed fuses
               only one of the two boundary kinds per layer (attention output or MLP output), the
               mixes the capture-time tuning may choose (decode_fused runs that tuning); decode_hd64 runs
               the TinyLlama attention shape (head_dim 64, KV heads replicated across ranks at 4 ranks).
Rank 0 prints one JSON summary; the exit code is non-zero on any failure.
"""
from __future__ import annotations

import argparse
import datetime
import hashlib
import json
import os
import random
import sys
import time
import traceback

import torch
import torch.distributed as dist

from ..ops.reference import TOL, dist_fused_allreduce_add_rmsnorm_ref, rel_err
from ..parallel import VARIANTS, TPCommTimeout, TPCommunicator


def digest(t: torch.Tensor) -> str:
    return hashlib.sha1(t.detach().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def same_everywhere(t: torch.Tensor) -> bool:
    d = [None] * dist.get_world_size()
    dist.all_gather_object(d, digest(t))
    return len(set(d)) == 1


class Checker:
    def __init__(self, rank):
        self.rank, self.fails, self.n = rank, [], 0

    def check(self, cond: bool, what: str):
        self.n += 1
        if not cond:
            self.fails.append(what)

    def all_ok(self) -> tuple[bool, list]:
        fails = [None] * dist.get_world_size()
        dist.all_gather_object(fails, self.fails)
        flat = [f"rank{r}: {m}" for r, fs in enumerate(fails) for m in fs]
        return not flat, flat


def inputs(rows, hidden, dtype, dev, seed):
    rank = dist.get_rank()
    g = torch.Generator(device=dev).manual_seed(seed * 100 + rank)
    x = torch.randn(rows, hidden, generator=g, device=dev).to(dtype)
    g2 = torch.Generator(device=dev).manual_seed(seed)  # replicated on every rank
    res = torch.randn(rows, hidden, generator=g2, device=dev).to(dtype)
    gamma = (1 + 0.1 * torch.randn(hidden, generator=g2, device=dev)).to(dtype)
    return x, res, gamma


# the cluster row-sum exchange form of the one-shot (passed the 2-GPU self-test on B200)
EXPERIMENTAL_VARIANTS = ["lamport_1sx"]


def functional(C: Checker, dev, world):
    variants = ["lamport_1s", "lamport_2s", "pull_1s", "pull_2s"] + EXPERIMENTAL_VARIANTS
    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        comm = TPCommunicator(dist.group.WORLD, device=dev, dtype=dtype, max_rows=128, max_hidden=8192)
        vs = variants + (["nvls_1s", "nvls_2s"] if comm.have_nvls else [])
        shapes = [(1, 8192), (3, 5120), (8, 4096), (64, 8192), (128, 2048)] if dtype != torch.float32 else \
            [(1, 4096), (7, 2048)]
        for v in vs:
            for rows, hidden in shapes:
                x, res0, gamma = inputs(rows, hidden, dtype, dev, seed=rows + hidden)
                ref_out, ref_h = dist_fused_allreduce_add_rmsnorm_ref(x, res0, gamma, 1e-6)
                res = res0.clone()
                out, res = comm.fused_allreduce_add_rmsnorm(x, res, gamma, 1e-6, variant=v)
                torch.cuda.synchronize()
                tol = 1e-5 if dtype == torch.float32 else TOL
                e1, e2 = rel_err(out, ref_out), rel_err(res, ref_h)
                C.check(e1 <= tol and e2 <= tol, f"{v} {dtype} [{rows},{hidden}] err {e1:.2e}/{e2:.2e}")
                C.check(same_everywhere(out) and same_everywhere(res), f"{v} {dtype} [{rows},{hidden}] ranks differ")
                ar = comm.all_reduce(x, variant=v)
                total = x.float().clone()
                dist.all_reduce(total)
                torch.cuda.synchronize()
                C.check(rel_err(ar, total) <= (1e-5 if dtype == torch.float32 else TOL), f"all_reduce {v} {dtype}")
        comm.check()
        if dtype == torch.bfloat16:
            w = torch.arange(16, device=dev, dtype=torch.int32) + 1000 * dist.get_rank()
            got = comm.all_gather_u32(w)
            torch.cuda.synchronize()
            C.check(all(torch.equal(got[r], torch.arange(16, device=dev, dtype=torch.int32) + 1000 * r)
                        for r in range(world)), "all_gather_u32")
            interleave(C, comm, dev, vs)
            late_rank(C, comm, dev)
        C.check(True, f"nvls available: {comm.have_nvls}")
        C.nvls = comm.have_nvls
        comm.close()


def interleave(C: Checker, comm: TPCommunicator, dev, vs):
    H, dtype = 5120, torch.bfloat16
    rng = random.Random(0)  # same sequence on every rank
    seq = [(rng.choice([1, 3, 8, 13, 40, 64, 128]), rng.choice([1, 2, 4, 8, 16]), rng.choice(vs)) for _ in range(60)]
    gamma = (1 + 0.1 * torch.randn(H, generator=torch.Generator(device=dev).manual_seed(7), device=dev)).to(dtype)
    for mode in ("eager", "graph"):
        graphs = {}
        if mode == "graph":
            for key in sorted(set(seq)):
                nt, nb, v = key
                xg = torch.zeros(nt, H, device=dev, dtype=dtype)
                rg = torch.zeros(nt, H, device=dev, dtype=dtype)
                og = torch.empty_like(xg)
                comm.fused_allreduce_add_rmsnorm(xg, rg, gamma, 1e-6, out=og, variant=v, blocks=nb)
                torch.cuda.synchronize()
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr):
                    comm.fused_allreduce_add_rmsnorm(xg, rg, gamma, 1e-6, out=og, variant=v, blocks=nb)
                graphs[key] = (gr, xg, rg, og)
            torch.cuda.synchronize()
            dist.barrier()
        bad = 0
        for i, (nt, nb, v) in enumerate(seq):
            x, res0, _ = inputs(nt, H, dtype, dev, seed=1000 + i)
            ref_out, ref_h = dist_fused_allreduce_add_rmsnorm_ref(x, res0, gamma, 1e-6)
            if mode == "eager":
                res = res0.clone()
                out, res = comm.fused_allreduce_add_rmsnorm(x, res, gamma, 1e-6, variant=v, blocks=nb)
            else:
                gr, xg, res, out = graphs[(nt, nb, v)]
                xg.copy_(x)
                res.copy_(res0)
                gr.replay()
            torch.cuda.synchronize()
            if rel_err(out, ref_out) > TOL or rel_err(res, ref_h) > TOL:
                bad += 1
        C.check(bad == 0, f"interleave {mode}: {bad}/60 wrong")
        del graphs
    comm.check()


def late_rank(C: Checker, comm: TPCommunicator, dev):
    x, res0, gamma = inputs(8, 8192, torch.bfloat16, dev, seed=5)
    ref_out, _ = dist_fused_allreduce_add_rmsnorm_ref(x, res0, gamma, 1e-6)
    for v in ("lamport_1s", "lamport_2s", "pull_2s"):
        torch.cuda.synchronize()
        dist.barrier()
        if dist.get_rank() == dist.get_world_size() - 1:
            time.sleep(0.2)  # the last rank launches 200 ms late; the others' kernels wait (bounded 1 s)
        out, _ = comm.fused_allreduce_add_rmsnorm(x, res0.clone(), gamma, 1e-6, variant=v)
        torch.cuda.synchronize()
        C.check(rel_err(out, ref_out) <= TOL, f"late rank {v}")
    comm.check()


def fault(C: Checker, dev, world):
    """Host-side fault injection: the last rank skips one call; nothing faults on the GPU."""
    comm = TPCommunicator(dist.group.WORLD, device=dev, dtype=torch.bfloat16, max_rows=16, max_hidden=4096,
                          timeout_ms=100, backend="ipc")
    C.check(not comm.have_nvls, "ipc heap must not have multicast")
    x, res0, gamma = inputs(4, 4096, torch.bfloat16, dev, seed=9)
    ref_out, _ = dist_fused_allreduce_add_rmsnorm_ref(x, res0, gamma, 1e-6)
    skipper = world - 1
    for v in ("lamport_1s", "lamport_2s", "pull_1s", "pull_2s"):
        torch.cuda.synchronize()
        dist.barrier()
        if dist.get_rank() != skipper:
            comm.fused_allreduce_add_rmsnorm(x, res0.clone(), gamma, 1e-6, variant=v)
        torch.cuda.synchronize()
        raised = False
        try:
            comm.check()
        except TPCommTimeout:
            raised = True
        C.check(raised == (dist.get_rank() != skipper), f"fault {v}: timeout reported={raised}")
        comm.reset()  # collective: host barrier, re-initialise every heap
        out, _ = comm.fused_allreduce_add_rmsnorm(x, res0.clone(), gamma, 1e-6, variant=v)
        torch.cuda.synchronize()
        comm.check()
        C.check(rel_err(out, ref_out) <= TOL, f"after reset {v}")
    comm.close()


def leave(C: Checker, dev, world, steps: int = 6, leave_at: int = 2):
    """A rank leaves the TP group between steps, with none of its kernels in flight: it posts its departure
    in the store instead of reaching the next step; the others learn of it in RankMonitor.sync() before
    they launch that step, so no kernel waits on the departed rank. Every rank then stays for the final
    host-side result exchange. CUDA-IPC heap, plain peer loads (no multicast object involved)."""
    from ..parallel.health import RankFailure, RankMonitor

    comm = TPCommunicator(dist.group.WORLD, device=dev, dtype=torch.bfloat16, max_rows=16, max_hidden=4096,
                          timeout_ms=1000, backend="ipc")
    mon = RankMonitor.from_default_group(prefix="selftest/leave", stale_s=60)
    mon.wait_joined(60)
    x, res0, gamma = inputs(4, 4096, torch.bfloat16, dev, seed=11)
    ref_out, _ = dist_fused_allreduce_add_rmsnorm_ref(x, res0, gamma, 1e-6)
    leaver, done, reason = world - 1, 0, ""
    for step in range(steps):
        if dist.get_rank() == leaver and step == leave_at:
            torch.cuda.synchronize()
            mon.leave()
            break
        try:
            mon.sync(60)
        except RankFailure as e:
            reason = str(e)
            break
        out, _ = comm.fused_allreduce_add_rmsnorm(x, res0.clone(), gamma, 1e-6, variant="lamport_1s")
        torch.cuda.synchronize()
        C.check(rel_err(out, ref_out) <= TOL, f"leave: step {step} result")
        done += 1
    C.check(done == leave_at, f"leave: rank stopped after {done} steps, expected {leave_at}")
    if dist.get_rank() != leaver:
        C.check("left the group" in reason, f"leave: departure not reported ({reason!r})")
    comm.check()  # no bounded wait ran out: nobody launched a call the leaver would not join
    comm.close()  # host-side teardown; every process, the leaver's too, is still alive


def stress(C: Checker, dev, world, calls: int = 120):
    """Memory-ordering stress: fused calls (variants and sizes in a seeded random order, the same on
    every rank) and layer boundaries while a side stream keeps the SMs busy with large GEMMs. Every call
    is checked against the fp32 NCCL oracle; the side load is bounded by a launch count."""
    comm = TPCommunicator(dist.group.WORLD, device=dev, dtype=torch.bfloat16, max_rows=64, max_hidden=8192)
    comm.prepare_fused_gemm(4096)
    rng = random.Random(1234)  # same sequence on every rank
    side = torch.cuda.Stream(dev)
    a = torch.randn(8192, 8192, device=dev, dtype=torch.bfloat16)
    vs = ["lamport_1s", "lamport_2s", "pull_1s", "pull_2s"] + EXPERIMENTAL_VARIANTS + \
        (["nvls_1s", "nvls_2s"] if comm.have_nvls else [])
    g = torch.Generator(device=dev).manual_seed(99 + dist.get_rank())
    w1 = (0.02 * torch.randn(4096, 1024, generator=g, device=dev)).bfloat16()
    w2 = (0.02 * torch.randn(384, 4096, generator=g, device=dev)).bfloat16()
    bad = 0
    for i in range(calls):
        with torch.cuda.stream(side):  # compute load overlapping the collective
            for _ in range(2):
                torch.mm(a, a)
        if rng.random() < 0.75:
            v, rows = rng.choice(vs), rng.choice([1, 3, 8, 17, 64])
            x, res0, gamma = inputs(rows, 8192, torch.bfloat16, dev, seed=i)
            ref_out, ref_h = dist_fused_allreduce_add_rmsnorm_ref(x, res0, gamma, 1e-6)
            res = res0.clone()
            out, res = comm.fused_allreduce_add_rmsnorm(x, res, gamma, 1e-6, variant=v)
            torch.cuda.synchronize()
            ok = rel_err(out, ref_out) <= TOL and rel_err(res, ref_h) <= TOL
        else:
            M = rng.choice([1, 5, 16])
            x = torch.randn(M, 1024, generator=g, device=dev).bfloat16()
            res0 = torch.randn(M, 4096, device=dev, generator=torch.Generator(device=dev).manual_seed(i)).bfloat16()
            gam = torch.ones(4096, device=dev, dtype=torch.bfloat16)
            y = (x.float() @ w1.float().t())
            dist.all_reduce(y)
            h = res0.float() + y
            ref = (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-5)) @ w2.float().t()
            res = res0.clone()
            comm.gemm_push(x, w1)
            z = comm.ar_norm_gemm(res, gam, w2, 1e-5)
            torch.cuda.synchronize()
            ok = rel_err(z, ref) <= TOL and rel_err(res, h) <= TOL
        bad += 0 if ok else 1
    side.synchronize()
    comm.check()
    C.check(bad == 0, f"stress: {bad} of {calls} calls wrong under concurrent GEMM load")
    comm.close()


def decode_check(C: Checker, dev, world, fused: bool = False, epilogues: bool = False, collective: str = "ours",
                 model: str = "tiny", kinds: tuple[bool, bool] | None = None):
    import math

    import torch.nn.functional as F

    from dataclasses import replace

    from ..models.llama import PRESETS, LlamaWeights, TPDecodeRunner
    from ..ops.reference import rope_tables

    cfg = replace(PRESETS[model], layers=2)
    full = LlamaWeights.full_random(cfg, device=dev, seed=3)
    w = LlamaWeights(cfg, dist.get_rank(), world, dev, full=full)
    comm = TPCommunicator(dist.group.WORLD, device=dev, dtype=torch.bfloat16, max_rows=8, max_hidden=cfg.hidden)
    car_group = dist.new_group(backend="gloo") if collective == "vllm" else None
    runner = TPDecodeRunner(cfg, w, comm, max_batch=4, max_seq=96, device=dev, nccl_group=dist.group.WORLD,
                            car_group=car_group,
                            fuse_boundary=fused, fuse_epilogues=epilogues, collective=collective,
                            tune_boundaries=kinds is None)
    if kinds is not None:  # a fixed mix of fused and separate boundaries instead of the timed choice
        runner.fuse_kinds[3] = kinds
    C.check(runner.fuse_boundary == fused, "layer-boundary fusion engaged as requested")
    prompts = torch.randint(0, cfg.vocab, (3, 29), generator=torch.Generator().manual_seed(1))
    first = runner.prefill(prompts)
    buf = runner.start(3, first, 29)
    runner.capture(3)
    D = cfg.head_dim

    def ref_logits(tokens):
        B, P = tokens.shape
        cos, sin = rope_tables(P, D, cfg.rope_theta, dev)
        c, sn = cos[None, :, None, :], sin[None, :, None, :]

        def rope(t):
            return torch.cat([t[..., :D // 2] * c - t[..., D // 2:] * sn, t[..., D // 2:] * c + t[..., :D // 2] * sn],
                             -1)

        x = full["embed"].float()[tokens.to(dev).long()]
        for L in full["layers"]:
            L = {k: v.float() for k, v in L.items()}
            h = F.rms_norm(x, (cfg.hidden,), L["ln1"], cfg.eps)
            qkv = h @ L["wqkv"].t() + (L["bqkv"] if "bqkv" in L else 0.0)
            q, k, v = qkv.split([cfg.heads * D, cfg.kv_heads * D, cfg.kv_heads * D], -1)
            q, k = rope(q.view(B, P, cfg.heads, D)), rope(k.view(B, P, cfg.kv_heads, D))
            a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                               v.view(B, P, cfg.kv_heads, D).transpose(1, 2), is_causal=True,
                                               enable_gqa=True, scale=1 / math.sqrt(D))
            x = x + a.transpose(1, 2).reshape(B, P, -1) @ L["wo"].t()
            h = F.rms_norm(x, (cfg.hidden,), L["ln2"], cfg.eps)
            g, u = (h @ L["wgu"].t()).chunk(2, -1)
            x = x + (F.silu(g) * u) @ L["wdown"].t()
        h = F.rms_norm(x[:, -1], (cfg.hidden,), full["final_norm"].float(), cfg.eps)
        return h @ full["lm_head"].float().t()

    toks = torch.cat([prompts, first.cpu()[:, None].long()], 1)
    V = cfg.vocab // world
    r = dist.get_rank()
    for step in range(3):
        runner.step(3)
        torch.cuda.synchronize()
        ref = ref_logits(toks)[:, r * V:(r + 1) * V]
        C.check(rel_err(buf["logits"], ref) < 2 ** -5,
                f"decode step {step} (fused={fused}) logits err {rel_err(buf['logits'], ref):.3e}")
        C.check(same_everywhere(buf["ids"]), f"decode step {step}: ranks disagree on tokens")
        toks = torch.cat([toks, buf["ids"].cpu()[:, None].long()], 1)
    runner.release_graphs()
    comm.check()
    comm.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--parts", default="functional,decode")
    a = ap.parse_args()
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    world, rank = dist.get_world_size(), dist.get_rank()
    C = Checker(rank)
    C.nvls = None
    err = ""
    t0 = time.time()
    try:
        for part in a.parts.split(","):
            {"functional": functional, "fault": fault, "leave": leave, "decode": decode_check, "stress": stress,
             "decode_fused": lambda C, dev, world: decode_check(C, dev, world, fused=True),
             "decode_fused_epi": lambda C, dev, world: decode_check(C, dev, world, fused=True, epilogues=True),
             "decode_nccl": lambda C, dev, world: decode_check(C, dev, world, collective="nccl"),
             "decode_vllm": lambda C, dev, world: decode_check(C, dev, world, collective="vllm"),
             # Qwen2.5-shaped attention: QKV bias, 5 query heads per KV head at 4 ranks
             "decode_qkv_bias": lambda C, dev, world: decode_check(C, dev, world, fused=True, model="tiny-qkv-bias"),
             "decode_mixed": lambda C, dev, world: [decode_check(C, dev, world, fused=True, kinds=k)
                                                    for k in ((True, False), (False, True))],
             # TinyLlama-shaped attention: head_dim 64, KV heads replicated when world > 2
             "decode_hd64": lambda C, dev, world: decode_check(C, dev, world, fused=True, model="tiny-hd64")
             }[part](C, dev, world)
    except Exception:
        err = traceback.format_exc()
        C.fails.append(err[-2000:])
    ok, fails = C.all_ok()
    if rank == 0:
        print(json.dumps(dict(ok=ok, world=world, parts=a.parts, checks=C.n, nvls=C.nvls, seconds=round(time.time() - t0, 1),
                              failures=fails[:20])), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
