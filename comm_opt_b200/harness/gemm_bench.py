"""Decode GEMM microbenchmark: our tcgen05 swap-AB kernel vs cuBLAS (torch.matmul) per shape.

    python -m comm_opt_b200.harness.gemm_bench [--shapes 70b-tp8,70b-tp1] [--batch 1,8,32,128]

Each measurement cycles through enough copies of the weight matrix that the working set exceeds
the 126 MB L2 (every call streams its weights from HBM, as in decode), times `iters` calls with CUDA
events after warm-up, and reports achieved HBM bandwidth (weight + activation + output bytes per
call / time) and its fraction of the measured copy bandwidth in MEASURED_PEAKS.json.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from ..models.gemm import gemm, pack_weight
from ..models.llama import PRESETS

L2_BYTES = 126 << 20


def shapes_for(name: str) -> list[tuple[str, int, int]]:
    model, tp = name.split("-tp")
    cfg, tp = PRESETS[model], int(tp)
    s = cfg.shard(tp)
    D, H = cfg.head_dim, cfg.hidden
    return [("qkv", (s["nq"] + 2 * s["nkv"]) * D, H), ("o", H, s["nq"] * D), ("gate_up", 2 * s["inter"], H),
            ("down", H, s["inter"]), ("lm_head", s["vocab"], H)]


def peak_hbm_gbs() -> float:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0  # no MEASURED_PEAKS.json: the earlier measurement of this pool (reported as "of fallback")


def time_fn(fn, iters: int) -> float:
    """Device time per call: `iters` calls captured in one CUDA graph (no host launch overhead),
    replayed after warm-up, timed with CUDA events."""
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1000.0 / iters


VARIANTS = {  # name -> gemm() keyword arguments
    "default": {},
    "pdl": dict(pdl=True),
    "small": dict(small_smem=True),
    "small_pdl": dict(small_smem=True, pdl=True),
    "tiles": dict(ctas=-1),  # one CTA per output tile (no split tiles)
    "tiles_small_pdl": dict(ctas=-1, small_smem=True, pdl=True),
    "cl2": dict(cluster_splits=2), "cl4": dict(cluster_splits=4), "cl8": dict(cluster_splits=8),
    "cl2_small_pdl": dict(cluster_splits=2, small_smem=True, pdl=True),
    "cl4_small_pdl": dict(cluster_splits=4, small_smem=True, pdl=True),
    "cl8_small_pdl": dict(cluster_splits=8, small_smem=True, pdl=True),
    "cl16_small_pdl": dict(cluster_splits=16, small_smem=True, pdl=True),
}


def variant_kwargs(v: str, N: int) -> tuple[dict, bool]:
    """gemm() keyword arguments of a variant name, and whether it runs on packed weights ("pk_" prefix:
    the same schedule on PackedWeight blocks; "_sw" suffix: a cluster schedule with the SwiGLU epilogue,
    output [M, N / 2], for the gate_up projection)."""
    packed = v.startswith("pk_") or v == "pk"
    sw = v.endswith("_sw")
    v = v[:-3] if sw else v
    base = v[3:] if v.startswith("pk_") else ("default" if v == "pk" else v)
    kw = dict(VARIANTS[base], **({"swiglu": True} if sw else {}))
    if kw.get("ctas") == -1:
        kw["ctas"] = (N + 127) // 128
    return kw, packed


def sweep(shape_sets: list[str], batches: list[int], variants: list[str], iters: int = 50, dev=None,
          ops: list[str] | None = None) -> list[dict]:
    """Time several launch variants of our kernel per shape (graph-captured, weights > L2)."""
    dev = dev or torch.device("cuda", 0)
    peak = peak_hbm_gbs()
    rows = []
    for sset in shape_sets:
        for name, N, K in shapes_for(sset):
            if ops and name not in ops:
                continue
            wbytes = N * K * 2
            copies = max(2, (2 * L2_BYTES) // wbytes + 1)
            ws = [torch.empty(N, K, dtype=torch.bfloat16, device=dev).normal_(0, 0.02) for _ in range(copies)]
            for M in batches:
                x = torch.randn(M, K, device=dev).to(torch.bfloat16)
                y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                nbytes = wbytes + (M * K + M * N) * 2
                row = dict(set=sset, op=name, M=M, N=N, K=K)
                for v in variants:
                    kw, packed = variant_kwargs(v, N)
                    sw = kw.get("swiglu", False)
                    if sw and name != "gate_up":
                        continue
                    wv = [pack_weight(w, interleave=64 if sw else 0) for w in ws] if packed else ws
                    yv = torch.empty(M, N // 2, device=dev, dtype=torch.bfloat16) if sw else y
                    t = time_fn(lambda i: gemm(x, wv[i % copies], yv, **kw), iters)
                    del wv
                    row[v] = round(t, 2)
                    row[v + "_frac"] = round((nbytes - (M * N // 2 * 2 if sw else 0)) / t / 1e3 / peak, 3)
                row["cublas"] = round(time_fn(lambda i: torch.matmul(x, ws[i % copies].t(), out=y), iters), 2)
                rows.append(row)
                print(json.dumps(row), flush=True)
            del ws
    return rows


def run(shape_sets: list[str], batches: list[int], iters: int = 50, dev=None) -> list[dict]:
    dev = dev or torch.device("cuda", 0)
    peak = peak_hbm_gbs()
    rows = []
    for sset in shape_sets:
        for name, N, K in shapes_for(sset):
            wbytes = N * K * 2
            copies = max(2, (2 * L2_BYTES) // wbytes + 1)
            ws = [torch.empty(N, K, dtype=torch.bfloat16, device=dev).normal_(0, 0.02) for _ in range(copies)]
            for M in batches:
                x = torch.randn(M, K, device=dev).to(torch.bfloat16)
                y = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
                nbytes = wbytes + (M * K + M * N) * 2
                t_cob = time_fn(lambda i: gemm(x, ws[i % copies], y), iters)
                t_cublas = time_fn(lambda i: torch.matmul(x, ws[i % copies].t(), out=y), iters)
                ref = x.float() @ ws[0].float().t()
                err = float((gemm(x, ws[0], y).float() - ref).abs().max() / ref.abs().max())
                rows.append(dict(set=sset, op=name, M=M, N=N, K=K, us_cob=round(t_cob, 2), us_cublas=round(t_cublas, 2),
                                 gbs_cob=round(nbytes / t_cob / 1e3, 1), frac_hbm_cob=round(nbytes / t_cob / 1e3 / peak, 3),
                                 speedup_vs_cublas=round(t_cublas / t_cob, 3), rel_err=err))
                print(json.dumps(rows[-1]), flush=True)
            del ws
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="70b-tp8,70b-tp1")
    ap.add_argument("--batch", default="1,8,32,128")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--out", default=None)
    ap.add_argument("--variants", default=None, help="comma list of launch variants to compare: " + ",".join(VARIANTS))
    ap.add_argument("--ops", default=None, help="only these projections (qkv,o,gate_up,down,lm_head)")
    a = ap.parse_args()
    if a.variants:
        rows = sweep(a.shapes.split(","), [int(b) for b in a.batch.split(",")], a.variants.split(","), a.iters,
                     ops=a.ops.split(",") if a.ops else None)
    else:
        rows = run(a.shapes.split(","), [int(b) for b in a.batch.split(",")], a.iters)
    if a.out:
        Path(a.out).write_text(json.dumps(rows, indent=1))


if __name__ == "__main__":
    main()
