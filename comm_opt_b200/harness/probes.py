"""Primitive probes: reduce-scatter by remote atomics (four `red` forms), push vs pull all-gather /
reduce-scatter primitives in steady state, the 128-byte line-atomicity premise test (`--line`), and SM
clock calibration.

    python -m comm_opt_b200.harness.probes --emulate 8                 (all ranks on one GPU)
    timeout -k 60 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \
        --master-port 29541 -m comm_opt_b200.harness.probes            (one rank per GPU, NVLink atomics)

For each variant and size: every rank adds its slice for owner d into d's accumulator, owners wait
for all arrivals (bounded), the accumulator is checked against the fp32 sum (relative error; f32 adds
are exact up to ordering, bf16x2 adds round on every arrival), and the kernel is timed with CUDA
events (max over ranks). The reference found 4-byte atomics too slow to build a reduce-scatter on
A100 (exp/M11_before_prototype/README.md:188); sm_100a adds 16-byte vector forms.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from .._ext import native

VARIANTS = {0: "red.f32", 1: "red.v4.f32", 2: "red.bf16x2", 3: "red.v4.bf16x2"}


def clock_mhz(device: int = 0, ns: int = 20_000_000) -> float:
    cycles, t = native().clock_calibration(ns, device)
    return cycles / t * 1000.0


def run_rs(world: int, n: int, variant: int, dev, emulate: bool, blocks: int = 64, reps: int = 5,
           group=None) -> dict:
    C = native()
    es = 4 if variant <= 1 else 2
    dt = torch.float32 if variant <= 1 else torch.bfloat16
    acc_bytes = (n * es + 4095) // 4096 * 4096
    region = acc_bytes + 4096
    rank = 0 if emulate else dist.get_rank(group)
    g = torch.Generator(device=dev).manual_seed(1234)
    if emulate:
        heap = torch.zeros(world * region, dtype=torch.uint8, device=dev)
        bases = [heap.data_ptr() + r * region for r in range(world)]
        x = (0.1 * torch.randn(world, world * n, generator=g, device=dev)).to(dt)
        mine = [heap[r * region: r * region + n * es].view(dt) for r in range(world)]
        zero = [heap]
    else:
        import torch.distributed._symmetric_memory as symm_mem

        heap = symm_mem.empty(region, dtype=torch.uint8, device=dev)
        hdl = symm_mem.rendezvous(heap, group or dist.group.WORLD)
        bases = list(hdl.buffer_ptrs)
        allx = (0.1 * torch.randn(world, world * n, generator=g, device=dev)).to(dt)
        x = allx[rank].contiguous()
        mine = [heap[:n * es].view(dt)]
        zero = [heap]
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    times = []
    for it in range(reps + 1):
        for z in zero:
            z.zero_()
        torch.cuda.synchronize()
        if not emulate:
            dist.barrier(group=group)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        x_rank_bytes = world * n * es if emulate else 0  # a real rank's x holds only its own slices
        C.rs_atomic_probe(bases, 0, acc_bytes, x, rank, n, variant, int(emulate), x_rank_bytes, blocks,
                          int(1e9), err)
        b.record()
        torch.cuda.synchronize()
        if it:
            times.append(a.elapsed_time(b) * 1000.0)
    src = x if emulate else allx
    if emulate:
        rels = []
        for d in range(world):
            ref = sum(src[r, d * n:(d + 1) * n].float() for r in range(world))
            rels.append(float((mine[d].float() - ref).abs().max() / ref.abs().max()))
        rel = max(rels)
    else:
        ref = sum(src[r, rank * n:(rank + 1) * n].float() for r in range(world))
        rel = float((mine[0].float() - ref).abs().max() / ref.abs().max())
    t = sorted(times)[len(times) // 2]
    if not emulate:
        tt = torch.tensor([t, rel, float(err.item())], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX, group=group)
        t, rel, e = [float(v) for v in tt.cpu()]
    else:
        e = float(err.item())
    return dict(variant=VARIANTS[variant], world=world, emulated=emulate, slice_bytes=n * es, us=round(t, 2),
                push_gbs=round((world - 1) * n * es / t / 1e3, 1), rel_err=rel, timeout=bool(e))


PRIM_MODES = {0: "ag_pull", 1: "ag_push", 2: "rs_pull", 3: "rs_push", 4: "rs_nvls", 5: "ag_nvls"}
NVLS_MODES = (4, 5)  # NVSwitch multicast (multimem.ld_reduce / multimem.st): real ranks with a multicast heap


def run_prim(world: int, n: int, mode: int, dev, emulate: bool, blocks: int = 64, threads: int = 256,
             graph_ops: int = 20, replays: int = 10, group=None, timeout_ms: float = 1000.0) -> dict:
    """Steady state (the reference's M13 'steady' mode): `graph_ops` launches per CUDA graph on buffers
    that are never cleared between launches; every word is checked against its (rank, index, epoch)
    hash inside the kernel. n = 32-bit words per rank (AG: n / world contributed, n gathered; RS: n
    contributed, n / world reduced). Returns per-op p50 us (max over ranks) and the mismatch count.
    The NVSwitch forms (modes 4, 5) need real ranks and a heap bound to a multicast object; without one
    the row says so instead of a time."""
    C = native()
    total, f_off, st_off, l_off, nv_off = C.prim_layout(world, n)
    if mode in NVLS_MODES and emulate:
        return dict(mode=PRIM_MODES[mode], world=world, emulated=True, words=n, skip="multicast needs real ranks")
    mc = 0
    rank = 0 if emulate else dist.get_rank(group)
    S = n // world
    if emulate:
        heap = torch.zeros(world * total, dtype=torch.uint8, device=dev)
        bases = [heap.data_ptr() + r * total for r in range(world)]
        for r in range(world):
            heap[r * total + l_off: (r + 1) * total].view(torch.int32).fill_(-2 ** 31)
    else:
        import torch.distributed._symmetric_memory as symm_mem

        heap = symm_mem.empty(total, dtype=torch.uint8, device=dev)
        heap.zero_()
        heap[l_off:].view(torch.int32).fill_(-2 ** 31)
        hdl = symm_mem.rendezvous(heap, group or dist.group.WORLD)
        bases = list(hdl.buffer_ptrs)
        mc = int(getattr(hdl, "multicast_ptr", 0) or 0)
        if mode in NVLS_MODES and not mc:  # every rank takes this branch alike (same heap kind)
            dist.barrier(group=group)
            return dict(mode=PRIM_MODES[mode], world=world, emulated=False, words=n, skip="no multicast object")
        torch.cuda.synchronize()
        dist.barrier(group=group)
    bad = torch.zeros(world if emulate else 1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    def call():
        C.prim_probe(bases, [f_off, st_off, l_off, nv_off], rank, n, mode, int(emulate), blocks, threads,
                     int(timeout_ms * 1e6), bad, err, mc)

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    if not emulate:
        dist.barrier(group=group)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(graph_ops):
            call()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(replays + 1)]
    g.replay()
    torch.cuda.synchronize()
    if not emulate:
        dist.barrier(group=group)
    ev[0].record()
    for i in range(replays):
        g.replay()
        ev[i + 1].record()
    torch.cuda.synchronize()
    times = sorted(ev[i].elapsed_time(ev[i + 1]) * 1000.0 / graph_ops for i in range(replays))
    t = times[len(times) // 2]
    nbad, nerr = float(bad.sum().item()), float(err.item())
    del g
    if not emulate:
        tt = torch.tensor([t, nbad, nerr], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX, group=group)
        t, nbad, nerr = [float(v) for v in tt.cpu()]
        dist.barrier(group=group)
    # NVLink bytes per GPU and call in the busier direction: (W - 1) slices for the peer forms; the whole
    # vector for the switch forms (ld_reduce pulls every GPU's part of every rank's slice through the
    # switch; multimem.st brings every slice, the own one included, back from the switch)
    moved = (world - 1) * S * 4 if mode not in NVLS_MODES else world * S * 4
    return dict(mode=PRIM_MODES[mode], world=world, emulated=emulate, words=n, us=round(t, 2),
                link_gbs=round(moved / t / 1e3, 1), bad_words=int(nbad), timeout=bool(nerr),
                calls=3 + graph_ops * (replays + 1))


LINE_MODES = {0: "atomic_add", 1: "store_4B", 2: "store_16B"}


def run_line(world: int, n_lines: int, mode: int, dev, emulate: bool, runs: int = 3, observer_blocks: int = 0,
             writer_blocks: int = 0, group=None, cpu_group=None, timeout_ms: float = 2000.0) -> dict:
    """Line-atomicity premise test (the reference's M8, exp/M8_ll128_atomic_a100/test_ll128_atomic.cu): rank 0
    observes its own buffer of n_lines 128-byte lines while ranks 1..W-1 write them over NVLink (emulate:
    every role as blocks of one launch on one GPU, L2 instead of NVLink). A violation is a line whose flag
    word says complete while another word does not match; `raced` counts lines the observer saw before they
    completed (with none, the run shows nothing either way). Store modes run `runs` launches on the same
    buffer with growing epochs; the atomic mode clears it before each launch."""
    C = native()
    target = 0
    rank = 0 if emulate else dist.get_rank(group)
    nbytes = n_lines * 128
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    if emulate:
        ob = observer_blocks or 16
        wb = writer_blocks or max(1, (sms - ob) // (world - 1))
        heap = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        bases = [heap.data_ptr()] * world
    else:
        import torch.distributed._symmetric_memory as symm_mem

        ob, wb = observer_blocks or sms, writer_blocks or 2 * sms
        heap = symm_mem.empty(nbytes, dtype=torch.uint8, device=dev)
        heap.zero_()
        bases = list(symm_mem.rendezvous(heap, group or dist.group.WORLD).buffer_ptrs)
    counters = torch.zeros(5, dtype=torch.int64, device=dev)

    def barrier():
        torch.cuda.synchronize()
        if not emulate:
            dist.barrier(group=cpu_group)  # host-only: an NCCL barrier would queue behind the observer

    rows = []
    for r in range(1, runs + 1):
        if mode == 0 and rank == target:
            heap.zero_()
        counters.zero_()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        C.line_probe(bases, nbytes, 0, n_lines, rank, target, mode, int(emulate), ob, wb, r, int(timeout_ms * 1e6),
                     counters, False)
        b.record()
        barrier()
        if rank == target:
            C.line_probe(bases, nbytes, 0, n_lines, rank, target, mode, int(emulate), ob, wb, r, 0, counters, True)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) if (emulate or rank != target) else 0.0
        vals = counters.cpu().tolist() + [ms]
        if not emulate:
            t = torch.tensor(vals, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=cpu_group)  # counters live on the target only
            vals = t.tolist()
        viol, raced, tmo, seen, final_bad, ms = vals
        per_writer = nbytes if mode == 0 else nbytes / (world - 1)
        rows.append(dict(run=r, violations=int(viol), raced_lines=int(raced), timeouts=int(tmo), observed=int(seen),
                         final_bad_lines=int(final_bad), writer_ms=round(ms, 3),
                         gbs_per_writer=round(per_writer / (ms * 1e-3) / 1e9, 1) if ms > 0 else None))
    del heap
    return dict(mode=LINE_MODES[mode], world=world, emulated=emulate, lines=n_lines, observer_blocks=ob,
                writer_blocks=wb, runs=rows, violations=sum(x["violations"] for x in rows),
                raced_lines=sum(x["raced_lines"] for x in rows), timeouts=sum(x["timeouts"] for x in rows),
                final_bad_lines=sum(x["final_bad_lines"] for x in rows))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--emulate", type=int, default=0, help="run W ranks in one launch on one GPU")
    ap.add_argument("--sizes", default="10240,81920,655360")
    ap.add_argument("--prim", action="store_true", help="push vs pull primitives instead of the atomic RS probe")
    ap.add_argument("--line", action="store_true", help="line-atomicity premise test instead of the atomic RS probe")
    ap.add_argument("--lines", type=int, default=1 << 20, help="--line: 128-byte lines in the observed buffer")
    ap.add_argument("--runs", type=int, default=3)
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    rows = []
    if a.emulate:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        world, rank = a.emulate, 0
    else:
        local = int(os.environ["LOCAL_RANK"])
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        world, rank = dist.get_world_size(), dist.get_rank()
    if a.line:
        cpu_group = None if a.emulate else dist.new_group(backend="gloo")
        for mode in LINE_MODES:
            r = run_line(world, a.lines, mode, dev, bool(a.emulate), runs=a.runs, cpu_group=cpu_group)
            rows.append(r)
            if rank == 0:
                print(json.dumps(r), flush=True)
    for n in ([] if a.line else [int(s) for s in a.sizes.split(",")]):
        for v in (PRIM_MODES if a.prim else VARIANTS):
            n_w = n // (4 * world) * 4 * world if a.prim else n
            r = run_prim(world, n_w, v, dev, bool(a.emulate)) if a.prim else run_rs(world, n, v, dev, bool(a.emulate))
            rows.append(r)
            if rank == 0:
                print(json.dumps(r), flush=True)
    if rank == 0:
        mhz = clock_mhz(dev.index)
        print(json.dumps(dict(clock_mhz=round(mhz, 1))), flush=True)
        if a.out:
            with open(a.out, "w") as f:
                json.dump(dict(rows=rows, clock_mhz=mhz), f, indent=1)
    if not a.emulate:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
