"""Where the time of one fused call goes, from the kernels' own phase stamps (%globaltimer, ns).

The reference splits a decode step into compute / exposed communication / waiting from profiler traces
(exp/M5_e2e_comm_share/traces.py:87-167) and restated vLLM's custom all-reduce with phase stamps
(exp/M11_before_prototype/car_timed.cu:34-47); this tool goes one level down, inside the fused collective
(with `--allreduce`, inside the plain all-reduce, whose pull variants share vLLM's phase structure):
every block of every call records start, inputs sent (or staged), barrier passed / owner slice reduced,
all peer data received and done. Per variant and token count it reports, as the max over ranks of the
per-rank mean over calls:

  sent / reduced / received / done : latest block's stamp - earliest block's start of the same call
  gap                              : next call's earliest start - this call's latest done, for calls
                                     back to back in one CUDA graph (launch + epoch hand-over cost)
  skew                             : spread of the calls' start stamps across ranks, reported only when
                                     the GPUs' %globaltimer clocks agree to within 1 ms (they are not
                                     synchronised across GPUs in general)
  op_us / op_us_stamped            : graph time per call without and with stamps (stamping overhead)

    timeout -k 60 600 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 \
        --master-addr 127.0.0.1 --master-port 29531 -m comm_opt_b200.harness.phase_profile \
        --variants lamport_1s,lamport_2s --tokens 1,8,64,512
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
from pathlib import Path

import torch
import torch.distributed as dist

from ..parallel import TPCommunicator
from ..utils.results import RunDir
from ..utils.stats import summary

PHASES = ("start", "sent", "reduced", "received", "done")


def graph_time_us(fn, ops: int, replays: int) -> tuple[torch.cuda.CUDAGraph, float]:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(ops):
            fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(replays + 1)]
    ev[0].record()
    for i in range(replays):
        g.replay()
        ev[i + 1].record()
    torch.cuda.synchronize()
    return g, summary([ev[i].elapsed_time(ev[i + 1]) * 1000.0 / ops for i in range(replays)])["p50"]


def decompose(stamps: torch.Tensor, epochs: list[int], blocks: int, ops: int) -> tuple[dict, list[int]]:
    """stamps: [cap, kMaxBlocks, phases] int64 of one rank; epochs: consecutive calls, `ops` per graph replay."""
    cap = stamps.shape[0]
    starts, ends, acc, gaps = [], [], {p: [] for p in PHASES[1:]}, []
    for e in epochs:
        blk = stamps[e % cap, :blocks]
        t0 = int(blk[:, 0].min())
        starts.append(t0)
        ends.append(int(blk[:, 4].max()))
        for i, ph in enumerate(PHASES[1:], start=1):
            col = blk[:, i]
            if int(col.min()) > 0:  # phase recorded by every block of this variant
                acc[ph].append((int(col.max()) - t0) / 1000.0)
    for k in range(len(epochs) - 1):
        if (k + 1) % ops:  # next call in the same replay
            gaps.append((starts[k + 1] - ends[k]) / 1000.0)
    out = {ph: (sum(v) / len(v) if v else None) for ph, v in acc.items()}
    out["gap"] = sum(gaps) / len(gaps) if gaps else None
    return out, starts


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--tokens", default="1,8,64,512")
    ap.add_argument("--variants", default="lamport_1s,lamport_2s")
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--graph-ops", type=int, default=20)
    ap.add_argument("--replays", type=int, default=10)
    ap.add_argument("--out-dir", default=None)
    ap.add_argument("--allreduce", action="store_true",
                    help="plain all-reduce (norm epilogue off): pull_1s / pull_2s then have the phase structure of "
                         "vLLM's one-stage / two-stage custom all-reduce (barrier, peer loads, barrier)")
    a = ap.parse_args()
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    cpu = dist.new_group(backend="gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    DT, H = getattr(torch, a.dtype), a.hidden
    tokens = [int(t) for t in a.tokens.split(",")]
    comm = TPCommunicator(dist.group.WORLD, device=dev, dtype=DT, max_rows=max(tokens), max_hidden=H)
    run = RunDir("phase_profile_ar" if a.allreduce else "phase_profile", Path(a.out_dir) if a.out_dir else None) \
        if rank == 0 else None
    if run:
        run.snapshot()
    cap = a.graph_ops * a.replays + 8
    gamma = torch.ones(H, dtype=DT, device=dev)
    rows = []
    for v in a.variants.split(","):
        for T in tokens:
            x = torch.randn(T, H, device=dev).to(DT)
            res = torch.randn(T, H, device=dev).to(DT)
            out = torch.empty_like(x)

            def fn():
                if a.allreduce:
                    comm.all_reduce(x, out, variant=v)
                else:
                    comm.fused_allreduce_add_rmsnorm(x, res, gamma, 1e-6, out=out, variant=v)

            err = ""
            try:
                comm.disable_stamps()
                dist.barrier(group=cpu)
                g, plain = graph_time_us(fn, a.graph_ops, a.replays)
                del g
                comm.enable_stamps(cap=cap)
                dist.barrier(group=cpu)
                g, stamped = graph_time_us(fn, a.graph_ops, a.replays)
                del g
                comm.check()
                last = comm.epochs()[0]
                epochs = list(range(last - a.graph_ops * a.replays + 1, last + 1))
                ph, starts = decompose(comm.stamps[0].cpu(), epochs, comm.last_choice.blocks, a.graph_ops)
            except Exception as e:  # recorded; every rank still takes the same collective steps below
                err, plain, stamped, ph, starts = f"{type(e).__name__}: {str(e)[:160]}", None, None, {}, []
            comm.disable_stamps()
            allr = [None] * world
            dist.all_gather_object(allr, (plain, stamped, ph, starts, err), group=cpu)
            if rank == 0:
                errs = next((r[4] for r in allr if r[4]), "")
                row = dict(variant=v, tokens=T, bytes=T * H * DT.itemsize, world=world, error=errs,
                           choice=comm.last_choice.__dict__ if comm.last_choice else None)
                if not errs:
                    row["op_us"] = max(r[0] for r in allr)
                    row["op_us_stamped"] = max(r[1] for r in allr)
                    for k in list(PHASES[1:]) + ["gap"]:
                        vals = [r[2].get(k) for r in allr if r[2].get(k) is not None]
                        row[k] = max(vals) if vals else None
                    n = min(len(r[3]) for r in allr)
                    skews = [max(r[3][i] for r in allr) - min(r[3][i] for r in allr) for i in range(n)]
                    sk = summary([s / 1000.0 for s in skews])["p50"] if skews else None
                    row["skew"] = sk if sk is not None and sk < 1000.0 else None
                rows.append(row)
                fmt = lambda k: "   -  " if row.get(k) is None else f"{row[k]:6.2f}"  # noqa: E731
                print(f"{v:11s} T{T:4d} op {fmt('op_us')} (stamped {fmt('op_us_stamped')})  sent {fmt('sent')} "
                      f"reduced {fmt('reduced')} received {fmt('received')} done {fmt('done')} gap {fmt('gap')} "
                      f"skew {fmt('skew')} {errs}", flush=True)
    if rank == 0:
        run.write_json("phases.json", dict(args=vars(a), world=world, comm=comm.describe(), rows=rows))
        print(json.dumps(dict(results=str(run.path))), flush=True)
    torch.cuda.synchronize()
    dist.barrier(group=cpu)
    comm.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
