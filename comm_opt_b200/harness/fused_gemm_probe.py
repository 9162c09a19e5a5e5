"""One-GPU probe of the layer-boundary kernels (gemm_push -> ar_norm_gemm) at Llama-70B TP=8 shapes with
the ranks emulated in one launch each: device time per call (CUDA events over a CUDA graph of K calls)
and a small, fixed workload for a profiler capture of one kernel.

    python -m comm_opt_b200.harness.fused_gemm_probe --world 2 --batch 8
    ncu --set full --clock-control none -k regex:k_ar_norm_gemm -s 4 -c 1 -o fg \
        python -m comm_opt_b200.harness.fused_gemm_probe --world 2 --batch 8 --iters 3

Emulated ranks share one GPU's HBM and SMs (each kernel runs every rank's CTAs), so times are per
emulated call, not per-rank latencies; the multi-GPU numbers come from harness/boundary_bench.py.
"""
from __future__ import annotations

import argparse
import json

import torch

from ..parallel import TPCommunicator


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--world", type=int, default=2)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--k1", type=int, default=3584)
    ap.add_argument("--hidden", type=int, default=8192)
    ap.add_argument("--n2", type=int, default=1280)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    W, M, K1, H, N2 = a.world, a.batch, a.k1, a.hidden, a.n2
    comm = TPCommunicator(emulate_world=W, device=dev, dtype=torch.bfloat16, max_rows=M, max_hidden=H)
    g = torch.Generator(device=dev).manual_seed(0)
    w1 = (0.02 * torch.randn(W, H, K1, generator=g, device=dev)).bfloat16()
    w2 = (0.02 * torch.randn(W, N2, H, generator=g, device=dev)).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).bfloat16()
    res = torch.randn(W, M, H, generator=g, device=dev).bfloat16()
    x = torch.randn(W, M, K1, generator=g, device=dev).bfloat16()
    out = torch.empty(W, M, N2, dtype=torch.bfloat16, device=dev)

    def call():
        comm.gemm_push(x, w1)
        comm.ar_norm_gemm(res, gamma, w2, 1e-5, out=out)

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(a.iters + 1)]
    ev[0].record()
    for i in range(a.iters):
        call()
        ev[i + 1].record()
    torch.cuda.synchronize()
    comm.check()
    us = sorted(ev[i].elapsed_time(ev[i + 1]) * 1000.0 for i in range(a.iters))
    print(json.dumps(dict(world=W, batch=M, k1=K1, hidden=H, n2=N2, p50_us=us[len(us) // 2], min_us=us[0],
                          plan_push=None, plan_consumer=comm.last_fused_gemm)))


if __name__ == "__main__":
    main()
