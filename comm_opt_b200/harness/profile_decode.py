"""Profiling driver: build a Llama-shaped runner and replay captured decode steps inside an NVTX
range named "decode", so a profiler can select exactly the decode kernels:

    python -m comm_opt_b200.harness.profile_decode --model 70b --layers 8 --batch 8 --steps 3
    ncu --nvtx --nvtx-include "decode/" --metrics gpu__time_duration.sum --clock-control none \
        --csv --log-file launches.csv python -m comm_opt_b200.harness.profile_decode ...

`--layers` shrinks the model for profiling only (every layer runs the same kernels).
"""
from __future__ import annotations

import argparse
from dataclasses import replace

import torch

from ..models.llama import PRESETS, LlamaWeights, TPDecodeRunner
from ..parallel import TPCommunicator


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="70b")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--gemm", default="cob")
    ap.add_argument("--eager", action="store_true")
    ap.add_argument("--l2-prefetch", type=int, default=0, help="weight tiles each GEMM prefetches into L2 while waiting")
    ap.add_argument("--gemm-timeline", action="store_true",
                    help="stamp every GEMM of the captured step (%%globaltimer) and print when each ran inside one "
                         "replay: the gaps between GEMMs hold the other kernels and the transitions")
    ap.add_argument("--attn-stages", type=int, default=0, help="attention KV ring depth (6: deep ring; 0: default)")
    ap.add_argument("--lin-cfg", action="append", default=[],
                    help="after tuning, force one projection's launch in every layer, e.g. "
                         "o=cluster_splits:2,small_smem:1 (ops qkv, o, gu, down; repeatable; 'tuned' keeps "
                         "the tuner's choices and prints them)")
    ap.add_argument("--tp-shape", type=int, default=1,
                    help="shard the weights this many ways (one GPU, the all-reduce replaced by add+RMSNorm) to "
                         "profile the per-rank kernels of a TP run")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if a.attn_stages:
        from ..ops import kernels as K

        K.set_attn_stages(a.attn_stages)
    cfg = replace(PRESETS[a.model], layers=a.layers)
    w = LlamaWeights(cfg, 0, a.tp_shape, dev, seed=0)
    comm = TPCommunicator(None, device=dev, dtype=torch.bfloat16, max_rows=max(8, a.batch), max_hidden=cfg.hidden)
    runner = TPDecodeRunner(cfg, w, comm, max_batch=a.batch, max_seq=a.prompt + a.steps + 64, device=dev, gemm=a.gemm,
                            l2_prefetch=a.l2_prefetch)
    if a.tp_shape > 1:  # per-rank shard shapes with the collective replaced by its local form
        runner.s = cfg.shard(a.tp_shape)
        runner.cache = type(runner.cache)(cfg, a.tp_shape, a.batch, a.prompt + a.steps + 64, dev)
    prompts = torch.randint(0, cfg.vocab, (a.batch, a.prompt), generator=torch.Generator().manual_seed(0))
    first = runner.prefill(prompts)
    runner.start(a.batch, first, a.prompt)
    stamps = None
    if a.lin_cfg and not a.eager:
        runner.tune(a.batch)
        print("tuned:", {op: runner.lin[(0, op)].cfg.get(a.batch) for op in ("qkv", "o", "down")},
              "gu fused:", runner.lin[(0, "gu")].fused.get(a.batch))
        for spec in a.lin_cfg:
            if spec == "tuned":  # keep the tuner's choices (a baseline run that prints them)
                continue
            op, kv = spec.split("=", 1)
            cfg_o = {k: int(v) for k, v in (item.split(":") for item in kv.split(",") if item)}
            for i in range(cfg.layers):
                lin = runner.lin[(i, op)]
                if op == "gu" and lin.fused.get(a.batch):
                    lin.fused[a.batch] = dict(cfg_o)
                else:
                    lin.cfg[a.batch] = dict(cfg_o)
        print("forced:", a.lin_cfg, {op: runner.lin[(0, op)].cfg.get(a.batch) for op in ("qkv", "o", "down")},
              "gu fused:", runner.lin[(0, "gu")].fused.get(a.batch))
    if a.gemm_timeline and not a.eager:
        from .._ext import native

        runner.tune(a.batch)  # the tuner's own launches are not stamped
        stride = 2048 * 16
        stamps = torch.zeros(1024 * stride, dtype=torch.int64, device=dev)
        native().set_gemm_stamps(stamps.data_ptr(), stride)
        runner.capture(a.batch, tune=False)
        n_total = native().gemm_stamp_launches()
        native().set_gemm_stamps(0, 0)
    elif not a.eager:
        runner.capture(a.batch, tune=not a.lin_cfg)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("decode")
    e0.record()
    for _ in range(a.steps):
        runner.step(a.batch, use_graph=not a.eager)
    e1.record()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    if stamps is not None:
        # the warm-up step and the captured step launch the same GEMMs: the captured ones are the second half
        n = n_total // 2
        stamps.zero_()
        runner.step(a.batch)
        torch.cuda.synchronize()
        st = stamps.view(1024, 2048, 16)[n:n_total].double()
        t0, prev_end, rows = None, None, []
        for i in range(n):
            s_i = st[i]
            ent = s_i[:, 0][s_i[:, 0] > 0]
            if ent.numel() == 0:
                continue
            beg, end = float(ent.min()), float(s_i[:, :10].max())
            t0 = beg if t0 is None else t0
            rows.append((i, (beg - t0) / 1e3, (end - beg) / 1e3, None if prev_end is None else (beg - prev_end) / 1e3,
                         int(ent.numel())))
            prev_end = end
        print("gemm  start_us  dur_us  gap_after_prev_us  ctas")
        for i, b, d, g, c in rows:
            print(f"{i:4d} {b:9.2f} {d:7.2f} {'' if g is None else f'{g:8.2f}':>10} {c:6d}")
        tot = sum(d for _, _, d, _, _ in rows)
        span = rows[-1][1] + rows[-1][2] if rows else 0.0
        print(f"gemm time {tot:.1f} us of a {span:.1f} us span ({len(rows)} GEMMs)")
    runner.release_graphs()
    print(f"ok kernels/step {runner.kernels_per_step.get(a.batch)} ms/step {e0.elapsed_time(e1) / a.steps:.3f} "
          f"(layers {a.layers}, tp-shape {a.tp_shape}, batch {a.batch}, l2 prefetch {a.l2_prefetch}, "
          f"attention stages {a.attn_stages or 'default'})")


if __name__ == "__main__":
    main()
