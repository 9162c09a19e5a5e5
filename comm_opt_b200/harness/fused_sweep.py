"""Fused all-reduce + residual + RMSNorm latency sweep (the reference's headline fused-op benchmark) on 2/4/8 GPUs.

    timeout -k 60 1800 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 \
        --master-addr 127.0.0.1 --master-port 29511 -m comm_opt_b200.harness.fused_sweep \
        --hidden 8192 --tokens 1,2,4,8,16,32,64,128,256,512

Per implementation and token count (message = tokens x hidden x 2 bytes, 16 KB - 8 MB at H 8192):
  1. correctness: seeded inputs, fp32 NCCL all-reduce oracle + fp32 residual/RMSNorm, relative error
     max|out - ref| / max|ref| <= 2^-5 on every rank (exp/M17_epoch_ab/bench_ab.py:137-164);
  2. timing: 5 eager calls, K calls captured in one CUDA graph, 3 warm replays, then R replays each
     bracketed by CUDA events; per-op time = replay time / K; for every replay the MAX over ranks
     is taken; p50 / p99 / mean over replays are reported (the reference kept only means).
Implementation order is shuffled with a recorded seed; a 2 s matmul warm-up brings clocks up first, and
the first (implementation, size) pair is measured twice with the first copy dropped (the reference's
discard-first rule, exp/M19_small_batch/bench_m19.py:249-252; `--discard-first 0` turns it off).
Results: results/<exp>/<timestamp>/ with env.txt, schedule.tsv, sweep.json (rank 0).
"""
from __future__ import annotations

import argparse
import contextlib
import datetime
import json
import os
import random
import time

import torch
import torch.distributed as dist

from ..baselines.fused import build
from ..ops.reference import TOL, dist_fused_allreduce_add_rmsnorm_ref, rel_err
from ..parallel import TPCommunicator
from ..utils.results import RunDir, gpu_state
from ..utils.stats import summary

DEFAULT_IMPLS = ("ours:auto,ours:lamport_1s,ours:lamport_1sx,ours:lamport_2s,ours:pull_1s,ours:pull_2s,ours:nvls_1s,"
                 "ours:nvls_2s,nccl_norm,vllm_car,trt_oneshot,trt_twoshot")


def warm_gpu(seconds: float, dev):
    a = torch.randn(4096, 4096, device=dev, dtype=torch.bfloat16)
    t0 = time.time()
    while time.time() - t0 < seconds:
        for _ in range(20):
            a = a @ a
            a = a / a.abs().max()
        torch.cuda.synchronize()
    return float(a.float().abs().mean())


def inputs(T, H, dtype, dev, seed, rank):
    g = torch.Generator(device=dev).manual_seed(seed * 1000 + rank + 1)
    x = torch.randn(T, H, generator=g, device=dev).to(dtype)
    g2 = torch.Generator(device=dev).manual_seed(seed * 1000 + 99)  # replicated
    res = torch.randn(T, H, generator=g2, device=dev).to(dtype)
    return x, res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--tokens", default="1,2,4,8,16,32,64,128,256,512")
    ap.add_argument("--impls", default=DEFAULT_IMPLS)
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--graph-ops", type=int, default=20)
    ap.add_argument("--replays", type=int, default=50)
    ap.add_argument("--eps", type=float, default=1e-6)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--warm-s", type=float, default=2.0)
    ap.add_argument("--nvlink", type=int, choices=[0, 1], default=0,
                    help="NVLink bytes per op from NVML's throughput counters around the timed replays (off by "
                         "default: the first 2-GPU sweep that read them aborted with host heap corruption)")
    ap.add_argument("--discard-first", type=int, choices=[0, 1], default=1,
                    help="measure the first (impl, tokens) config twice and drop the first copy")
    ap.add_argument("--exp", default="fused_sweep")
    ap.add_argument("--out-dir", default=None, help="base directory of results/ (default: repo results/)")
    ap.add_argument("--ts", default=None)
    a = ap.parse_args()

    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
    cpu_group = dist.new_group(backend="gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    DT = getattr(torch, a.dtype)
    H = a.hidden
    tokens = [int(t) for t in a.tokens.split(",")]
    maxT = max(tokens)
    from pathlib import Path

    run = RunDir(a.exp, Path(a.out_dir) if a.out_dir else None, a.ts) if rank == 0 else None
    if run:
        run.snapshot()
    comm = TPCommunicator(dist.group.WORLD, device=dev, dtype=DT, max_rows=maxT, max_hidden=H)
    impls, skipped = build(a.impls.split(","), comm=comm, rank=rank, world=world, max_rows=maxT, hidden=H, dtype=DT,
                           device=dev, cpu_group=cpu_group)
    gamma = (1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(7))).to(DT).to(dev)
    order = list(impls)
    random.Random(a.seed).shuffle(order)
    ctr = None
    if a.nvlink:
        try:
            from ..utils.nvlink import NvlinkCounters

            ctr = NvlinkCounters(torch.cuda.current_device())
            ctr = ctr if ctr.available else None
        except Exception as e:  # NVML missing or no NVLink: rows carry no byte counts
            print(f"rank {rank}: NVLink counters unavailable ({type(e).__name__}: {e})", flush=True)
            ctr = None
    warm_gpu(a.warm_s, dev)
    rows, n = [], 0
    plan = [(impl, T, False) for impl in order for T in tokens]
    if a.discard_first and plan:
        plan.insert(0, (plan[0][0], plan[0][1], True))  # first config measured twice, first copy dropped
    for impl, T, discard in plan:
        t_start, state = time.time(), gpu_state() if rank == 0 else ""
        reason = impl.available(T, H)
        reasons = [None] * world
        dist.all_gather_object(reasons, reason, group=cpu_group)
        reason = next((r for r in reasons if r), "")
        err, rel, times, link = "", float("nan"), [], {}
        if not reason:
            try:
                # ---- correctness on fresh inputs
                x, res0 = inputs(T, H, DT, dev, a.seed + T, rank)
                ref_out, ref_h = dist_fused_allreduce_add_rmsnorm_ref(x, res0, gamma, a.eps)
                res = res0.clone()
                fn = impl.make(x.clone(), res, gamma, a.eps)
                torch.cuda.synchronize()
                dist.barrier(group=cpu_group)
                out = fn()
                torch.cuda.synchronize()
                rel = rel_err(out, ref_out)
                if impl.residual_rows == "all":
                    rel = max(rel, rel_err(res, ref_h))
                else:  # rows owned by this rank (the reference keeps the residual sharded)
                    rp = -(-T // world)
                    r0, r1 = min(T, rank * rp), min(T, (rank + 1) * rp)
                    if r1 > r0:
                        rel = max(rel, rel_err(res[r0:r1], ref_h[r0:r1]))
                # ---- timing under graph replay
                x, res = inputs(T, H, DT, dev, a.seed + T + 1, rank)
                fn = impl.make(x, res, gamma, a.eps)
                for _ in range(5):
                    fn()
                torch.cuda.synchronize()
                dist.barrier(group=cpu_group)
                g = torch.cuda.CUDAGraph()
                with impl.capture_ctx():
                    with torch.cuda.graph(g):
                        for _ in range(a.graph_ops):
                            fn()
                for _ in range(3):
                    g.replay()
                torch.cuda.synchronize()
                dist.barrier(group=cpu_group)
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.replays + 1)]
                with (ctr.measure() if ctr else contextlib.nullcontext({})) as link:
                    ev[0].record()
                    for i in range(a.replays):
                        g.replay()
                        ev[i + 1].record()
                    torch.cuda.synchronize()
                times = [ev[i].elapsed_time(ev[i + 1]) * 1000.0 / a.graph_ops for i in range(a.replays)]
                del g
                if hasattr(comm, "check") and impl.name.startswith("ours"):
                    comm.check()
            except Exception as e:  # recorded per row; other rows continue
                err = f"{type(e).__name__}: {str(e)[:200]}"
        gathered = [None] * world
        dist.all_gather_object(gathered, (times, rel, err, link), group=cpu_group)
        if rank == 0:
            per_replay = [max(g[0][i] for g in gathered) for i in range(a.replays)] if all(
                len(g[0]) == a.replays for g in gathered) else []
            worst = max((g[1] for g in gathered if g[1] == g[1]), default=float("nan"))
            errs = next((g[2] for g in gathered if g[2]), "")
            s = summary(per_replay) if per_replay else {}
            row = dict(impl=impl.name, world=world, dtype=a.dtype, hidden=H, tokens=T, bytes=T * H * DT.itemsize,
                       p50_us=s.get("p50"), p99_us=s.get("p99"), mean_us=s.get("mean"),
                       per_rank_p50=[summary(g[0])["p50"] if g[0] else None for g in gathered],
                       max_rel_err=worst, correct=bool(worst == worst and worst <= TOL), skip=reason, error=errs,
                       variant=(comm.last_choice.__dict__ if impl.name.startswith("ours") and comm.last_choice else None))
            ops = a.replays * a.graph_ops
            if all(g[3].get("tx_bytes") is not None for g in gathered):
                row["nvlink_tx_bytes_per_op"] = max(g[3]["tx_bytes"] for g in gathered) / ops
                row["nvlink_rx_bytes_per_op"] = max(g[3]["rx_bytes"] for g in gathered) / ops
            if not discard:
                rows.append(row)
            print(f"{impl.name:16s} w{world} T{T:4d} {row['bytes'] >> 10:6d}KB p50 {row['p50_us'] or float('nan'):8.2f} us "
                  f"p99 {row['p99_us'] or float('nan'):8.2f} err {worst:.1e} {reason or errs}"
                  f"{' (discarded)' if discard else ''}", flush=True)
            run.schedule(n, f"{impl.name}_T{T}" + ("_discard" if discard else ""), t_start, time.time() - t_start,
                         0 if not errs else 1, state)
            n += 1
    if rank == 0:
        run.write_json("sweep.json", dict(args=vars(a), world=world, order=[i.name for i in order], skipped=skipped,
                                          comm=comm.describe(), rows=rows))
        print(json.dumps(dict(results=str(run.path), skipped=skipped)), flush=True)
    for impl in impls:
        try:
            impl.close()
        except Exception:
            pass
    torch.cuda.synchronize()
    dist.barrier(group=cpu_group)
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
