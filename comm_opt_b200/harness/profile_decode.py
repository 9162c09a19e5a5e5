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
    ap.add_argument("--tp-shape", type=int, default=1,
                    help="shard the weights this many ways (one GPU, the all-reduce replaced by add+RMSNorm) to "
                         "profile the per-rank kernels of a TP run")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = replace(PRESETS[a.model], layers=a.layers)
    w = LlamaWeights(cfg, 0, a.tp_shape, dev, seed=0)
    comm = TPCommunicator(None, device=dev, dtype=torch.bfloat16, max_rows=max(8, a.batch), max_hidden=cfg.hidden)
    runner = TPDecodeRunner(cfg, w, comm, max_batch=a.batch, max_seq=a.prompt + a.steps + 64, device=dev, gemm=a.gemm)
    if a.tp_shape > 1:  # per-rank shard shapes with the collective replaced by its local form
        runner.s = cfg.shard(a.tp_shape)
        runner.cache = type(runner.cache)(cfg, a.tp_shape, a.batch, a.prompt + a.steps + 64, dev)
    prompts = torch.randint(0, cfg.vocab, (a.batch, a.prompt), generator=torch.Generator().manual_seed(0))
    first = runner.prefill(prompts)
    runner.start(a.batch, first, a.prompt)
    if not a.eager:
        runner.capture(a.batch)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("decode")
    e0.record()
    for _ in range(a.steps):
        runner.step(a.batch, use_graph=not a.eager)
    e1.record()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    runner.release_graphs()
    print(f"ok kernels/step {runner.kernels_per_step.get(a.batch)} ms/step {e0.elapsed_time(e1) / a.steps:.3f} "
          f"(layers {a.layers}, tp-shape {a.tp_shape}, batch {a.batch})")


if __name__ == "__main__":
    main()
