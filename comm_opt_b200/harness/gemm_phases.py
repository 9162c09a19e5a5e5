"""Phase timeline of the decode GEMM from in-kernel %globaltimer stamps (one B200).

    python -m comm_opt_b200.harness.gemm_phases --shapes 70b-tp8 --batch 8 [--variants default,cl4_small_pdl]

For each projection shape and launch variant the kernel runs `--runs` times with L2 flushed before
every launch (weights come from HBM, as in decode); each CTA stamps its entry, set-up, the issue of its
first weight tiles, the dependency wait, its last load, its first landed stage, its last MMA, its
last accumulator and the end of its epilogue. Printed per phase (ns after the earliest CTA entry):
min / median / max over CTAs of the median run, plus the derived streaming rate per CTA (its weight
bytes over first-stage-landed .. last-MMA) and the whole kernel span next to the CUDA-event time of a
graph of back-to-back launches. The point is to see where a short GEMM spends its time: start-up
latency, weight streaming, or the tail.
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch

from .._ext import native
from ..models.gemm import gemm, pack_weight
from .gemm_bench import L2_BYTES, shapes_for, time_fn, variant_kwargs

PHASES = ("entry", "setup", "weights_issued", "pdl_wait", "last_load", "first_full", "last_mma", "acc_ready",
          "epi_done", "end")
SLOTS = 16


def timeline(stamps: torch.Tensor, ctas: int) -> dict:
    s = stamps[:ctas, :len(PHASES)].double()
    t0 = s[:, 0].min()
    out = {}
    for i, name in enumerate(PHASES):
        col = s[:, i]
        col = col[col > 0] - t0
        if col.numel():
            v = sorted(col.tolist())
            out[name] = (round(v[0]), round(v[len(v) // 2]), round(v[-1]))
    return out


def measure(op, N, K, M, variant, runs, dev):
    kw, packed = variant_kwargs(variant, N)
    w = torch.empty(N, K, dtype=torch.bfloat16, device=dev).normal_(0, 0.02)
    ref = None
    if packed:
        w0 = w
        w = pack_weight(w0)
    x = torch.randn(M, K, device=dev).to(torch.bfloat16)
    y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    stamps = torch.zeros(4096, SLOTS, dtype=torch.int64, device=dev)
    C = native()
    lines = []
    C.set_gemm_stamps(stamps.data_ptr())
    try:
        for _ in range(runs):
            stamps.zero_()
            flush.zero_()
            gemm(x, w, y, **kw)
            torch.cuda.synchronize()
            ctas = int((stamps[:, 0] > 0).sum())
            lines.append((timeline(stamps, ctas), ctas, stamps[:ctas].clone()))
    finally:
        C.set_gemm_stamps(0)
    spans = [tl["end"][2] for tl, _, _ in lines]
    med = sorted(range(runs), key=lambda i: spans[i])[runs // 2]
    tl, ctas, st = lines[med]
    per_cta_bytes = N * K * 2 / ctas
    stream_ns = (st[:, 6] - st[:, 5]).double().clamp_min(1)
    rate = sorted((per_cta_bytes / stream_ns).tolist())  # bytes/ns = GB/s
    if packed:  # the packed launch computes the same product as the row-major weight
        ref = x.float() @ w0.float().t()
        err = float((gemm(x, w, y, **kw).float() - ref).abs().max() / ref.abs().max())
        assert err < 2 ** -6, f"packed weights: relative error {err}"
    copies = max(2, (2 * L2_BYTES) // (N * K * 2) + 1)
    wc = [w] + [(pack_weight if packed else (lambda t: t))(torch.empty(N, K, dtype=torch.bfloat16, device=dev)
                                                          .normal_(0, 0.02)) for _ in range(copies - 1)]
    ev_us = time_fn(lambda i: gemm(x, wc[i % copies], y, **kw), 20)
    return dict(op=op, M=M, N=N, K=K, variant=variant, ctas=ctas, span_ns=tl["end"][2], event_us=round(ev_us, 2),
                phases_ns=tl, stream_gbs_per_cta=dict(min=round(rate[0], 1), med=round(rate[len(rate) // 2], 1),
                                                     max=round(rate[-1], 1)),
                stream_gbs_total=round(N * K * 2 / statistics.median(stream_ns.tolist()), 1))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="70b-tp8")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--variants", default="default")
    ap.add_argument("--ops", default=None)
    ap.add_argument("--runs", type=int, default=5)
    ap.add_argument("--out-dir", default=None, help="base directory of results/ (default: the repository's)")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rows = []
    for name, N, K in shapes_for(a.shapes):
        if a.ops and name not in a.ops.split(","):
            continue
        for v in a.variants.split(","):
            rows.append(measure(name, N, K, a.batch, v, a.runs, dev))
            print(json.dumps(rows[-1]), flush=True)
    from pathlib import Path

    from ..utils.results import RunDir

    run = RunDir("gemm_phases", Path(a.out_dir) if a.out_dir else None)
    run.snapshot()
    run.write_json("phases.json", dict(args=vars(a), rows=rows))
    print(run.path)


if __name__ == "__main__":
    main()
