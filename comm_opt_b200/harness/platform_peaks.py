"""Platform peaks of a B200 node, measured and committed as a record that the analyzers read.

    python -m comm_opt_b200.harness.platform_peaks [--gib 1] [--reps 10]

One process, every visible GPU (no torchrun). Measured with CUDA events after a warm-up, best of
`--reps`:

* hbm_copy_gbs: device-local copy of `--gib` GiB (read + write bytes / time), per GPU;
* peer_copy_gbs: GPU 0 -> GPU j copy of `--gib` GiB through the copy engines (cudaMemcpyPeer via
  torch), bytes / time, for every peer j: the per-direction NVLink figure;
* peer_bidir_gbs: GPU 0 <-> GPU 1 at once (two streams), bytes per direction / time;
* fanout_gbs: GPU 0 -> every peer at once, total bytes leaving GPU 0 / time.

Writes results/platform/<timestamp>/link.json (with env.txt). `comm_opt_b200.utils.peaks.link_gbs()`
returns the median peer_copy_gbs of the newest committed record: the NVLink denominator of every
roofline fraction (fused op, layer boundary), instead of a constant in the code.
"""
from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch

from ..utils.results import RunDir


def _time(fn, reps: int, streams) -> float:
    """Best elapsed seconds of `fn` over `reps` runs: events on the first stream, all streams joined."""
    best = float("inf")
    for _ in range(reps):
        for s in streams:
            s.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        start.record(streams[0])
        for s in streams[1:]:
            s.wait_event(start)
        fn()
        for s in streams[1:]:
            ev = torch.cuda.Event()
            ev.record(s)
            streams[0].wait_event(ev)
        stop.record(streams[0])
        stop.synchronize()
        best = min(best, start.elapsed_time(stop) / 1e3)
    return best


def measure(gib: float = 1.0, reps: int = 10) -> dict:
    n = torch.cuda.device_count()
    nbytes = int(gib * (1 << 30))
    out = dict(gpus=n, bytes=nbytes, reps=reps, name=torch.cuda.get_device_name(0))
    # bf16 elements, as the driver's own HBM copy measurement
    bufs = [torch.empty(nbytes // 2, dtype=torch.bfloat16, device=f"cuda:{d}") for d in range(n)]
    recv = [torch.empty(nbytes // 2, dtype=torch.bfloat16, device=f"cuda:{d}") for d in range(n)]
    streams = [torch.cuda.Stream(device=d) for d in range(n)]
    hbm = []
    for d in range(n):
        def copy_local(d=d):
            with torch.cuda.device(d), torch.cuda.stream(streams[d]):
                recv[d].copy_(bufs[d], non_blocking=True)
        copy_local()
        hbm.append(2 * nbytes / _time(copy_local, reps, [streams[d]]) / 1e9)
    out["hbm_copy_gbs"] = [round(v, 1) for v in hbm]
    if n < 2:
        return out
    peer = {}
    for j in range(1, n):
        def p2p(j=j):
            with torch.cuda.device(0), torch.cuda.stream(streams[0]):
                recv[j].copy_(bufs[0], non_blocking=True)
        p2p()
        peer[j] = nbytes / _time(p2p, reps, [streams[0]]) / 1e9
    out["peer_copy_gbs"] = {str(j): round(v, 1) for j, v in peer.items()}
    out["peer_copy_gbs_median"] = round(statistics.median(peer.values()), 1)

    def bidir():
        with torch.cuda.device(0), torch.cuda.stream(streams[0]):
            recv[1].copy_(bufs[0], non_blocking=True)
        with torch.cuda.device(1), torch.cuda.stream(streams[1]):
            recv[0].copy_(bufs[1], non_blocking=True)
    bidir()
    out["peer_bidir_gbs"] = round(nbytes / _time(bidir, reps, [streams[0], streams[1]]) / 1e9, 1)

    chunk = nbytes // 2 // (n - 1) // 128 * 128  # elements per peer
    fan = [torch.cuda.Stream(device=0) for _ in range(n - 1)]

    def fanout():
        for j in range(1, n):
            with torch.cuda.device(0), torch.cuda.stream(fan[j - 1]):
                recv[j][:chunk].copy_(bufs[0][:chunk], non_blocking=True)
    fanout()
    out["fanout_gbs"] = round(2 * chunk * (n - 1) / _time(fanout, reps, fan) / 1e9, 1)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gib", type=float, default=1.0)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--out-dir", default=None, help="base directory instead of results/")
    a = ap.parse_args(argv)
    res = measure(a.gib, a.reps)
    run = RunDir("platform", Path(a.out_dir) if a.out_dir else None)
    run.snapshot()
    run.write_json("link.json", res)
    print(json.dumps(res), flush=True)
    print(run.path)


if __name__ == "__main__":
    main()
