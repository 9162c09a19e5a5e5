"""Flagship benchmark: Llama-3-70B-shaped tensor-parallel greedy decode (the reference's headline TP=8 decode metric).

    python bench.py --gpus N --steps K --warmup W          (N > 1: launched by torch.distributed.run)

One timed step = one decode step of the whole batch (every sequence emits one token): embedding,
80 layers of our tcgen05 GEMMs / RoPE + paged-KV append / paged GQA attention / SiLU*mul and the
fused all-reduce + residual + RMSNorm kernel at both row-parallel outputs, LM head and a
distributed greedy argmax. The step is one CUDA graph replay. Metric: decode ms per token
(per step) of the whole job, device-timed with CUDA events, max over ranks; strong scaling (the
model and batch are fixed while N grows). Every step streams the full weight set (141 GB / N)
from HBM, far larger than the 126 MB L2, so no L2 flush is needed between steps.

`e2e` repeats the measurement through the public API `TPDecodeRunner.decode`, which copies each
step's input token ids from pinned host memory and reads the produced ids back to the host.

`--impl reference` runs the reference implementation; it is not an installable project (no
setup.py / pyproject.toml), so the arm prints an `unavailable` line.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=128)
    p.add_argument("--warmup", type=int, default=8)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--model", default="70b")
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--prompt", type=int, default=2048)
    p.add_argument("--gemm", choices=["cob", "torch"], default="cob")
    p.add_argument("--collective", choices=["ours", "nccl", "vllm"], default="ours",
                   help="nccl: the same runner with NCCL all-reduce + add/RMSNorm kernel (baseline decode step); "
                        "vllm: vLLM custom all-reduce + vLLM fused_add_rms_norm (the reference's baseline stack)")
    p.add_argument("--fuse-epilogues", type=int, choices=[0, 1], default=1,
                   help="with fused boundaries: SiLU * up and RoPE + KV append in the consumer GEMMs where they "
                        "have a geometry for them (with --tune-boundaries, kept only where measured faster)")
    p.add_argument("--fuse-boundary", type=int, choices=[0, 1], default=1,
                   help="fuse o_proj/down_proj -> all-reduce + RMSNorm -> next GEMM (TP > 1; 0 = separate "
                        "GEMM, fused all-reduce + RMSNorm kernel, GEMM)")
    p.add_argument("--tune-boundaries", type=int, choices=[0, 1], default=1,
                   help="with fused boundaries: time each fused / separate choice of the two boundary kinds at "
                        "capture and keep the fastest (0 = both fused)")
    p.add_argument("--l2-prefetch", type=int, default=0,
                   help="weight tiles each GEMM prefetches into L2 beyond its ring while it waits (0 = none)")
    p.add_argument("--e2e-steps", type=int, default=None)
    p.add_argument("--layers", type=int, default=None, help="override the layer count (debug only; invalid for bench)")
    p.add_argument("--out", default=None, help="also write the JSON line to this file")
    return p.parse_args()


class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices: list[int]):
        self.indices = indices
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", ",".join(map(str, self.indices))], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        return self.summarize(self.rows)

    @staticmethod
    def summarize(rows: list[list[str]]) -> dict:
        """Median SM clock, max clock, active throttle reasons over nvidia-smi rows of QUERY."""
        mhz, mx, reasons, power = [], [], set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                mhz.append(float(r[1]))
                mx.append(float(r[2]))
                power.append(float(r[3]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        mhz.sort()
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(mhz), "power_w_max": max(power) if power else None}


def reference_arm(args):
    line = {"impl": "reference",
            "unavailable": "the reference (allennnnnz/comm_opt) is not an installable project (pip install of its "
                           "source tree fails: 'Neither setup.py nor pyproject.toml found') and has no decode runner "
                           "of its own: its only decode path, exp/M5_e2e_comm_share/infer.py, drives the vLLM engine "
                           "on a Hugging Face checkpoint and tokenizer from the hub cache, which this offline box "
                           "does not have; its fused kernel is compared in harness/fused_sweep.py (ref_m16nf)"}
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(line), flush=True)


def result_line(args, cfg, world: int, ms: float, ms_e2e: float, e2e_steps: int, setup_s: float, clocks, runner) -> dict:
    """The driver's JSON line: device-timed ms per decode step (max over ranks), the end-to-end figure
    through TPDecodeRunner.decode, our kernel launches in the timed region, and the clock record."""
    B, P, K, W = args.batch, args.prompt, args.steps, args.warmup
    weights_gb = cfg.params * 2 / 1e9
    return {
        "metric": "llama3_70b_tp_decode_ms_per_token" if args.model in ("70b", "llama3-70b") else
        f"{cfg.name}_tp_decode_ms_per_token",
        "value": round(ms, 4),
        "unit": "ms/token",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms, 4),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: uniform-random prompt token ids (seed 1234), random-init weights N(0, 0.02)",
        "config": {"model": cfg.name + ("" if args.layers is None else f"-L{cfg.layers}-INVALID"),
                   "global_batch": B, "seq_len": P, "decode_tokens_timed": K, "parallelism": f"tp{world}",
                   "gemm": args.gemm, "collective": args.collective, "fuse_boundary": runner.fuse_boundary,
                   "fuse_epilogues": runner.fuse_boundary and runner.fuse_epilogues,
                   "fuse_fallback": runner.fuse_error[:200] or None,
                   "fused_boundaries": (dict(zip(("attention_out", "mlp_out"), runner.fuse_kinds.get(B, (True, True))),
                                             epilogues=dict(zip(("swiglu", "rope_kv"),
                                                                runner.fused_epilogues_used(B))),
                                             step_ms_by_choice=runner.boundary_times.get(B))
                                        if runner.fuse_boundary else None),
                   "gate_up_swiglu_epilogue": (runner.lin[(0, "gu")].kernels(B) == 1
                                               if args.gemm == "cob" else False),
                   "tokens_per_s": round(B * 1000.0 / ms, 1), "l2_prefetch_tiles": args.l2_prefetch,
                   "l2": f"no flush: each step streams the full weight set ({weights_gb:.0f} GB / {world} GPUs) "
                         ">> 126 MB L2",
                   "setup_s": round(setup_s, 1)},
        "e2e": {"value": round(ms_e2e, 4), "unit": "ms/token", "h2d_bytes_per_step": B * 4,
                "d2h_bytes_per_step": B * 4, "steps": e2e_steps, "api": "TPDecodeRunner.decode"},
        "gpu_launches": runner.kernels_per_step[B] * K,
        "kernels_per_step": runner.kernels_per_step[B],
        "clocks": clocks,
    }


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch
    import torch.distributed as dist

    from comm_opt_b200.models.llama import PRESETS, LlamaWeights, TPDecodeRunner
    from comm_opt_b200.parallel import TPCommunicator

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    group = None
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        group = dist.group.WORLD

    cfg = PRESETS[args.model]
    if args.layers:
        from dataclasses import replace

        cfg = replace(cfg, layers=args.layers)
    B, P, K, W = args.batch, args.prompt, args.steps, args.warmup
    E = args.e2e_steps if args.e2e_steps is not None else max(8, min(K, 64))
    max_seq = P + 1 + W + K + E + 2 * W + 16
    t0 = time.time()
    weights = LlamaWeights(cfg, rank, world, dev, seed=0)
    comm = TPCommunicator(group, device=dev, dtype=torch.bfloat16, max_rows=max(B, 8), max_hidden=cfg.hidden)
    car_group = dist.new_group(backend="gloo") if args.collective == "vllm" and world > 1 else None
    runner = TPDecodeRunner(cfg, weights, comm, max_batch=B, max_seq=max_seq, device=dev, gemm=args.gemm,
                            nccl_group=group, car_group=car_group, fuse_boundary=bool(args.fuse_boundary),
                            fuse_epilogues=bool(args.fuse_epilogues), collective=args.collective,
                            tune_boundaries=bool(args.tune_boundaries), l2_prefetch=args.l2_prefetch)
    prompts = torch.randint(0, cfg.vocab, (B, P), generator=torch.Generator().manual_seed(1234))
    first = runner.prefill(prompts)
    runner.start(B, first, P)
    runner.capture(B)
    torch.cuda.synchronize()
    setup_s = time.time() - t0

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    # ---------------- device-timed decode steps (graph replays)
    for _ in range(W):
        runner.step(B)
    barrier()
    phys = [int(x) for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip().isdigit()]
    sampler = ClockSampler([phys[i] if i < len(phys) else i for i in range(world)]) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.5)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    start.record()
    for _ in range(K):
        runner.step(B)
    end.record()
    torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end) / K
    clocks = sampler.stop() if sampler else None
    comm.check()

    # ---------------- end to end through the public decode API (pinned H2D ids, D2H ids)
    host_in = torch.empty(B, dtype=torch.int32).pin_memory()
    host_out = torch.empty(B, dtype=torch.int32).pin_memory()
    host_in.copy_(runner.graphs[B][1]["ids"].cpu())
    for _ in range(W):
        runner.decode(B, host_in, host_out)
        host_in.copy_(host_out)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(E):
        runner.decode(B, host_in, host_out)
        host_in.copy_(host_out)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    ms_e2e = e0.elapsed_time(e1) / E
    comm.check()

    stats = torch.tensor([ms, ms_e2e], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    ms, ms_e2e = [float(v) for v in stats.cpu()]
    if rank == 0:
        line = result_line(args, cfg, world, ms, ms_e2e, E, setup_s, clocks, runner)
        s = json.dumps(line)
        print(s, flush=True)
        if args.out:
            Path(args.out).write_text(s + "\n")
    runner.release_graphs()
    del runner
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
