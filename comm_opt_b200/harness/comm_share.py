"""Communication share of TP decode (the reference's M5 measurement, exp/M5_e2e_comm_share/infer.py with
traces.py), for this library's runner: every rank profiles `steps` graph-replayed decode steps,
writes a Chrome trace, and rank 0 decomposes them (harness/traces.py).

    timeout -k 60 900 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \
        --master-port 29531 -m comm_opt_b200.harness.comm_share --model 70b --layers 8 --batch 8 --out-dir traces/
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
from dataclasses import replace
from pathlib import Path

import torch
import torch.distributed as dist

from ..models.llama import PRESETS, LlamaWeights, TPDecodeRunner
from ..parallel import TPCommunicator
from .traces import decompose


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="70b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--out-dir", default="results/traces")
    ap.add_argument("--fuse-boundary", type=int, choices=[0, 1], default=1)
    a = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    group = None
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        group = dist.group.WORLD
    rank = dist.get_rank() if world > 1 else 0
    cfg = PRESETS[a.model] if a.layers is None else replace(PRESETS[a.model], layers=a.layers)
    w = LlamaWeights(cfg, rank, world, dev, seed=0)
    comm = TPCommunicator(group, device=dev, dtype=torch.bfloat16, max_rows=max(8, a.batch), max_hidden=cfg.hidden)
    runner = TPDecodeRunner(cfg, w, comm, max_batch=a.batch, max_seq=a.prompt + a.steps + 64, device=dev,
                            nccl_group=group, fuse_boundary=bool(a.fuse_boundary))
    prompts = torch.randint(0, cfg.vocab, (a.batch, a.prompt), generator=torch.Generator().manual_seed(0))
    first = runner.prefill(prompts)
    runner.start(a.batch, first, a.prompt)
    runner.capture(a.batch)
    for _ in range(3):
        runner.step(a.batch)
    torch.cuda.synchronize()
    out = Path(a.out_dir)
    out.mkdir(parents=True, exist_ok=True)
    acts = [torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA]
    with torch.profiler.profile(activities=acts) as prof:
        for _ in range(a.steps):
            with torch.profiler.record_function("decode_step"):
                runner.step(a.batch)
                torch.cuda.synchronize()
    path = out / f"trace_rank{rank}.json"
    prof.export_chrome_trace(str(path))
    if world > 1:
        dist.barrier()
    if rank == 0:
        rows = decompose(sorted(out.glob("trace_rank*.json")), "decode_step")
        share = sum(r["exposed_comm_us"] for r in rows) / max(1e-9, sum(r["wall_us"] for r in rows))
        fused = sum(r.get("fused_us", 0.0) for r in rows) / max(1e-9, sum(r["wall_us"] for r in rows))
        print(json.dumps(dict(model=cfg.name, layers=cfg.layers, tp=world, batch=a.batch, steps=a.steps,
                              fuse_boundary=runner.fuse_boundary, exposed_comm_share=round(share, 4),
                              fused_gemm_collective_share=round(fused, 4),
                              mean_wall_us=sum(r["wall_us"] for r in rows) / max(1, len(rows)))), flush=True)
    runner.release_graphs()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
