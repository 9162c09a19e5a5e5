"""Collective characterisation sweep (the reference's M0 baseline with nccl-tests, exp/M0_baseline/run.sh;
JSON rows as loaded by exp/lib/nccljson.py:9-33), built on torch.distributed/NCCL because nccl-tests and
MPI are not installed here.

    timeout -k 60 900 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \
        --master-port 29521 -m comm_opt_b200.harness.collectives --colls all_reduce,all_gather --begin 8 --end 64M

Per collective and size: `warmup` untimed iterations, then `iters` iterations each bracketed by CUDA
events (or, with --graph, K iterations captured in one CUDA graph, as nccl-tests -G); the time of an
iteration is the MAX over ranks. Reported per size: p50/p99/mean time, algorithm bandwidth
(size / time) and bus bandwidth with the nccl-tests correction factors (all_reduce 2(n-1)/n,
all_gather / reduce_scatter / alltoall (n-1)/n, broadcast / sendrecv 1), and a correctness flag
(`nwrong` = 0 when the result matches the expected value).
Environment variants (e.g. NCCL_ALGO, NCCL_PROTO, NCCL_NVLS_ENABLE, NCCL_MIN_NCHANNELS) are passed as
environment variables by the experiment runner (harness/runner.py).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import time

import torch
import torch.distributed as dist

from ..utils.stats import summary

BUS_FACTOR = {
    "all_reduce": lambda n: 2 * (n - 1) / n,
    "all_gather": lambda n: (n - 1) / n,
    "reduce_scatter": lambda n: (n - 1) / n,
    "alltoall": lambda n: (n - 1) / n,
    "broadcast": lambda n: 1.0,
    "sendrecv": lambda n: 1.0,
}


def parse_size(s: str) -> int:
    s = s.strip().upper()
    mult = {"K": 1 << 10, "M": 1 << 20, "G": 1 << 30}
    return int(float(s[:-1]) * mult[s[-1]]) if s[-1] in mult else int(s)


def make_op(coll: str, nbytes: int, dtype, dev, rank: int, world: int):
    """Returns (fn, check) for one collective of `nbytes` (the per-rank buffer size, nccl-tests -b/-e)."""
    es = torch.tensor([], dtype=dtype).element_size()
    n = max(world, nbytes // es // world * world) if coll in ("all_gather", "reduce_scatter", "alltoall") else \
        max(1, nbytes // es)
    x = torch.full((n,), float(rank + 1), dtype=dtype, device=dev)
    if coll == "all_reduce":
        def fn():
            x.fill_(rank + 1)
            dist.all_reduce(x)
        expect = world * (world + 1) / 2
        return fn, lambda: bool((x == expect).all())
    if coll == "all_gather":
        out = torch.empty(n, dtype=dtype, device=dev)
        xs = x[: n // world]

        def fn():
            dist.all_gather_into_tensor(out, xs)
        return fn, lambda: bool(all((out[r * (n // world):(r + 1) * (n // world)] == r + 1).all() for r in range(world)))
    if coll == "reduce_scatter":
        out = torch.empty(n // world, dtype=dtype, device=dev)

        def fn():
            dist.reduce_scatter_tensor(out, x)
        return fn, lambda: bool((out == world * (world + 1) / 2).all())
    if coll == "alltoall":
        out = torch.empty(n, dtype=dtype, device=dev)

        def fn():
            dist.all_to_all_single(out, x)
        return fn, lambda: bool(all((out[r * (n // world):(r + 1) * (n // world)] == r + 1).all() for r in range(world)))
    if coll == "broadcast":
        def fn():
            dist.broadcast(x, src=0)
        return fn, lambda: bool((x == 1).all())
    if coll == "sendrecv":
        out = torch.empty(n, dtype=dtype, device=dev)
        peer_to, peer_from = (rank + 1) % world, (rank - 1) % world

        def fn():
            ops = [dist.P2POp(dist.isend, x, peer_to), dist.P2POp(dist.irecv, out, peer_from)]
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        return fn, lambda: bool((out == peer_from + 1).all())
    raise ValueError(coll)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--colls", default="all_reduce,all_gather,reduce_scatter,alltoall,broadcast,sendrecv")
    ap.add_argument("--begin", default="8", help="smallest per-rank buffer (nccl-tests -b)")
    ap.add_argument("--end", default="256M", help="largest per-rank buffer (nccl-tests -e)")
    ap.add_argument("--factor", type=int, default=2)
    ap.add_argument("--iters", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--graph", type=int, default=0, help="capture K iterations in one CUDA graph (nccl-tests -G K)")
    ap.add_argument("--dtype", default="float32")
    ap.add_argument("--out", default=None, help="JSON output path (rank 0)")
    ap.add_argument("--device", default="cuda", choices=["cuda", "cpu"], help="cpu: gloo back end (tests)")
    a = ap.parse_args()
    local = int(os.environ["LOCAL_RANK"])
    on_gpu = a.device == "cuda"
    if on_gpu:
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
    else:
        dev = torch.device("cpu")
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
        a.graph = 0
    cpu = dist.new_group(backend="gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    dtype = getattr(torch, a.dtype)
    sizes, s = [], parse_size(a.begin)
    while s <= parse_size(a.end):
        sizes.append(s)
        s *= a.factor
    results = []
    for coll in a.colls.split(","):
        for nbytes in sizes:
            fn, check = make_op(coll, nbytes, dtype, dev, rank, world)
            for _ in range(a.warmup):
                fn()
            sync = torch.cuda.synchronize if on_gpu else (lambda: None)
            sync()
            ok = check()
            times = []
            if a.graph:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for _ in range(a.graph):
                        fn()
                g.replay()
                torch.cuda.synchronize()
            dist.barrier(group=cpu)
            per = a.graph or 1
            if on_gpu:
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.iters + 1)]
                ev[0].record()
                for i in range(a.iters):
                    if a.graph:
                        g.replay()
                    else:
                        fn()
                    ev[i + 1].record()
                torch.cuda.synchronize()
                times = [ev[i].elapsed_time(ev[i + 1]) * 1000.0 / per for i in range(a.iters)]
            else:
                times = []
                for i in range(a.iters):
                    t0 = time.perf_counter()
                    fn()
                    times.append((time.perf_counter() - t0) * 1e6)
            allt = [None] * world
            dist.all_gather_object(allt, (times, ok), group=cpu)
            if rank == 0:
                per_iter = [max(t[0][i] for t in allt) for i in range(a.iters)]
                st = summary(per_iter)
                algbw = nbytes / st["mean"] / 1e3  # GB/s (bytes / us / 1e3)
                row = dict(size=nbytes, coll=coll, world=world, time_us=st["mean"], p50_us=st["p50"], p99_us=st["p99"],
                           cv_pct=100.0 * (sum((t - st["mean"]) ** 2 for t in per_iter) / len(per_iter)) ** 0.5 /
                           st["mean"], algbw=algbw, busbw=algbw * BUS_FACTOR[coll](world),
                           nwrong=0 if all(t[1] for t in allt) else 1, graph=a.graph)
                results.append(row)
                print(f"{coll:15s} {nbytes:>12d} B  {st['p50']:9.2f} us  busbw {row['busbw']:8.2f} GB/s "
                      f"{'' if row['nwrong'] == 0 else 'WRONG'}", flush=True)
            if a.graph:
                del g
    if rank == 0:
        nccl = ".".join(map(str, torch.cuda.nccl.version())) if on_gpu else "gloo"
        doc = dict(version=f"torch {torch.__version__} nccl {nccl}", world=world, args=vars(a),
                   env={k: v for k, v in os.environ.items() if k.startswith("NCCL_")},
                   date=time.strftime("%Y-%m-%dT%H:%M:%S"), results=results)
        if a.out:
            with open(a.out, "w") as f:
                json.dump(doc, f, indent=1)
    dist.barrier(group=cpu)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
