"""Plain all-reduce bake-off: this package's kernels (norm epilogue off) against the all-reduces a
decode engine could use instead, timed identically inside CUDA graphs.

Capability of the reference's M6 bench (exp/M6_allreduce_bakeoff/bench_torch.py:21-122: torch NCCL,
vLLM custom all-reduce, PyTorch SymmetricMemory one-shot / two-shot; 1 KB - 8 MB; K all-reduces per
graph; error against an fp32 all-reduce of the same inputs), plus SymmetricMemory's NVSwitch multicast
forms (multimem one-shot and multimem all-reduce), which the reference's A100 system could not run, and
NCCL timed eagerly as well as in graphs (`torch_nccl@eager`; the reference's "NCCL eager" column,
exp/M6_allreduce_bakeoff/README.md:93-101). Per (implementation, size): one eager call
on seeded inputs checked against the fp32 sum, then 5 eager calls, K calls captured in one graph,
3 warm replays and R timed replays; the per-op time of a replay is its time / K, the MAX over ranks is
taken per replay, and p50 / p99 / mean over replays are reported (the reference reported the mean of
all replays per rank). The message is shaped [rows, hidden] with hidden = min(elements, 8192).

    timeout -k 60 900 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 \
        --master-addr 127.0.0.1 --master-port 29541 -m comm_opt_b200.harness.allreduce_bakeoff
"""
from __future__ import annotations

import argparse
import contextlib
import datetime
import json
import os
import random
import time
from pathlib import Path

import torch
import torch.distributed as dist

from ..parallel import TPCommunicator
from ..utils.results import RunDir, gpu_state
from ..utils.stats import summary

DEFAULT_IMPLS = ("ours:auto,ours:lamport_1s,ours:lamport_2s,ours:nvls_2s,torch_nccl,torch_nccl@eager,vllm_car,"
                 "symm_one_shot,symm_two_shot,symm_multimem,symm_multimem_one_shot")
EAGER = "@eager"  # suffix: time K eager calls per replay instead of a graph (the reference's "NCCL eager")
HIDDEN = 8192


def shape_of(nbytes: int, esize: int) -> tuple[int, int]:
    n = nbytes // esize
    h = min(n, HIDDEN)
    return max(1, n // h), h


class Bakeoff:
    """Builds (fn, capture context, reason-if-unavailable) for every implementation and size."""

    def __init__(self, impls, comm, cpu_group, dev, dtype, max_bytes):
        self.comm, self.cpu, self.dev, self.dt = comm, cpu_group, dev, dtype
        self.group_name = dist.group.WORLD.group_name
        self.car = self.symm = None
        self.skipped = {}
        if "vllm_car" in impls:
            try:
                from vllm.distributed.device_communicators.custom_all_reduce import CustomAllreduce

                self.car = CustomAllreduce(cpu_group, dev, max_size=max_bytes * 2)
                if self.car.disabled:
                    self.skipped["vllm_car"], self.car = "vLLM custom all-reduce disabled here", None
            except Exception as e:  # recorded, the other implementations still run
                self.skipped["vllm_car"] = f"{type(e).__name__}: {str(e)[:200]}"
        if any(i.startswith("symm_") for i in impls):
            try:
                import torch.distributed._symmetric_memory as symm_mem

                self.symm = symm_mem.empty(max_bytes // dtype.itemsize, dtype=dtype, device=dev)
                symm_mem.rendezvous(self.symm, group=dist.group.WORLD)
            except Exception as e:
                for i in impls:
                    if i.startswith("symm_"):
                        self.skipped[i] = f"{type(e).__name__}: {str(e)[:200]}"

    def available(self, impl: str, nbytes: int) -> str:
        impl = impl.removesuffix(EAGER)
        if impl in self.skipped:
            return self.skipped[impl]
        if impl == "vllm_car" and not self.car.should_custom_ar(torch.empty(nbytes // self.dt.itemsize, dtype=self.dt,
                                                                            device=self.dev)):
            return "vLLM declines this size"
        if impl.startswith("symm_") and self.dt != torch.bfloat16:
            return "SymmetricMemory one/two-shot are bf16 only"
        if impl.startswith("ours:"):
            v = impl.split(":", 1)[1]
            rows, h = shape_of(nbytes, self.dt.itemsize)
            hv = h * self.dt.itemsize // 16
            if v.endswith("_2s") and (hv % self.comm.world or hv % 32):
                return "hidden not divisible for two-shot"
            if v.startswith("nvls") and not self.comm.have_nvls:
                return "no NVSwitch multicast"
        return ""

    def make(self, impl: str, x: torch.Tensor):
        """x: this rank's input (flat). Returns (fn -> result tensor, capture context factory)."""
        impl = impl.removesuffix(EAGER)
        n = x.numel()
        if impl.startswith("ours:"):
            rows, h = shape_of(n * x.element_size(), x.element_size())
            xi, out, v = x.view(rows, h), torch.empty(rows, h, dtype=x.dtype, device=x.device), impl.split(":", 1)[1]
            return (lambda: self.comm.all_reduce(xi, out, variant=v).view(-1)), contextlib.nullcontext
        if impl == "torch_nccl":
            buf = x.clone()

            def fn():
                buf.copy_(x)  # in place: restart from the input so repeated calls stay finite
                dist.all_reduce(buf)
                return buf
            return fn, contextlib.nullcontext
        if impl == "vllm_car":
            return (lambda: self.car.custom_all_reduce(x)), self.car.capture
        s = self.symm[:n]
        s.copy_(x)
        if impl == "symm_one_shot":
            return (lambda: torch.ops.symm_mem.one_shot_all_reduce(s, "sum", self.group_name)), contextlib.nullcontext
        if impl == "symm_multimem_one_shot":  # NVSwitch multicast load-reduce (NVLS), one shot
            return (lambda: torch.ops.symm_mem.multimem_one_shot_all_reduce(s, "sum", self.group_name)), \
                contextlib.nullcontext
        if impl == "symm_multimem":  # NVLS reduce-scatter + multicast store, in place

            def mm():
                s.copy_(x)
                torch.ops.symm_mem.multimem_all_reduce_(s, "sum", self.group_name)
                return s
            return mm, contextlib.nullcontext

        def two():
            s.copy_(x)
            torch.ops.symm_mem.two_shot_all_reduce_(s, "sum", self.group_name)
            return s
        return two, contextlib.nullcontext

    def close(self):
        if self.car is not None:
            self.car.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--impls", default=DEFAULT_IMPLS)
    ap.add_argument("--min-bytes", type=int, default=1 << 10)
    ap.add_argument("--max-bytes", type=int, default=8 << 20)
    ap.add_argument("--graph-ops", type=int, default=20)
    ap.add_argument("--replays", type=int, default=20)
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--out-dir", default=None)
    a = ap.parse_args()
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
    cpu = dist.new_group(backend="gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    DT = getattr(torch, a.dtype)
    sizes, s = [], a.min_bytes
    while s <= a.max_bytes:
        sizes.append(s)
        s *= 2
    impls = a.impls.split(",")
    rmax, hmax = shape_of(a.max_bytes, DT.itemsize)
    comm = TPCommunicator(dist.group.WORLD, device=dev, dtype=DT, max_rows=rmax, max_hidden=hmax)
    bk = Bakeoff(impls, comm, cpu, dev, DT, a.max_bytes)
    run = RunDir("allreduce_bakeoff", Path(a.out_dir) if a.out_dir else None) if rank == 0 else None
    if run:
        run.snapshot()
    random.Random(a.seed).shuffle(impls)
    rows, n_job = [], 0
    for impl in impls:
        for nbytes in sizes:
            t0, state = time.time(), gpu_state() if rank == 0 else ""
            reasons = [None] * world
            dist.all_gather_object(reasons, bk.available(impl, nbytes), group=cpu)
            reason = next((r for r in reasons if r), "")
            err, rel, times = "", float("nan"), []
            if not reason:
                try:
                    n = nbytes // DT.itemsize
                    g = torch.Generator(device=dev).manual_seed(a.seed * 1000 + rank + 1)
                    src = torch.randn(n, generator=g, device=dev).to(DT)
                    exact = src.float()
                    dist.all_reduce(exact)
                    fn, ctx = bk.make(impl, src)
                    torch.cuda.synchronize()
                    dist.barrier(group=cpu)
                    out = fn()
                    torch.cuda.synchronize()
                    rel = float((out.float() - exact).abs().max() / exact.abs().max())
                    for _ in range(5):
                        fn()
                    torch.cuda.synchronize()
                    dist.barrier(group=cpu)
                    if impl.endswith(EAGER):  # K eager calls stand in for one graph replay
                        def replay():
                            for _ in range(a.graph_ops):
                                fn()
                        graph = None
                    else:
                        graph = torch.cuda.CUDAGraph()
                        with ctx():
                            with torch.cuda.graph(graph):
                                for _ in range(a.graph_ops):
                                    fn()
                        replay = graph.replay
                    for _ in range(3):
                        replay()
                    torch.cuda.synchronize()
                    dist.barrier(group=cpu)
                    ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.replays + 1)]
                    ev[0].record()
                    for i in range(a.replays):
                        replay()
                        ev[i + 1].record()
                    torch.cuda.synchronize()
                    times = [ev[i].elapsed_time(ev[i + 1]) * 1000.0 / a.graph_ops for i in range(a.replays)]
                    del graph
                    if impl.startswith("ours:"):
                        comm.check()
                except Exception as e:  # recorded per row; every rank still takes the gather below
                    err = f"{type(e).__name__}: {str(e)[:200]}"
            gathered = [None] * world
            dist.all_gather_object(gathered, (times, rel, err), group=cpu)
            if rank == 0:
                ok = all(len(g[0]) == a.replays for g in gathered)
                per = [max(g[0][i] for g in gathered) for i in range(a.replays)] if ok else []
                st = summary(per) if per else {}
                worst = max((g[1] for g in gathered if g[1] == g[1]), default=float("nan"))
                errs = next((g[2] for g in gathered if g[2]), "")
                row = dict(impl=impl, world=world, dtype=a.dtype, bytes=nbytes, p50_us=st.get("p50"),
                           p99_us=st.get("p99"), mean_us=st.get("mean"), max_rel_err=worst,
                           correct=bool(worst == worst and worst <= 2 ** -5), skip=reason, error=errs,
                           busbw_gbs=(2 * (world - 1) / world * nbytes / st["p50"] / 1e3) if st else None)
                rows.append(row)
                print(f"{impl:16s} w{world} {nbytes >> 10:6d}KB p50 {row['p50_us'] or float('nan'):8.2f} us "
                      f"err {worst:.1e} {reason or errs}", flush=True)
                run.schedule(n_job, f"{impl}_{nbytes}", t0, time.time() - t0, 1 if errs else 0, state)
                n_job += 1
    if rank == 0:
        run.write_json("bakeoff.json", dict(args=vars(a), world=world, order=impls, skipped=bk.skipped,
                                            comm=comm.describe(), rows=rows))
        print(json.dumps(dict(results=str(run.path), skipped=bk.skipped)), flush=True)
    bk.close()
    torch.cuda.synchronize()
    dist.barrier(group=cpu)
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
