"""Communication share of a training step: the reference's end-to-end training measurement
(exp/M5_e2e_comm_share/run_train.py:14-40, titan_recipes.py:31-75, analyze_train.py:38-83) on this
package's TP x FSDP trainer (models/train.py) instead of torchtitan.

Per launch: `warmup` steps, `steps` timed steps (CUDA events around each step, the total taken as the
max over ranks; this unprofiled step time is the denominator of every share), then `profile` steps under
the torch profiler with one Chrome trace per rank. Rank 0 splits the profiled steps
(harness/traces.py:breakdown) into compute, the compute slowdown caused by overlap, exposed transfer,
other time (CPU, waiting, idle) and exposed time per collective type, and writes summary.json beside the
traces. Every step copies its token batch from pinned host memory and reads the loss back, as a data
loader and a logger would.

    timeout -k 60 1800 python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \
        --master-port 29541 -m comm_opt_b200.harness.train_share --model 8b --tp 4 --out-dir results/train_share/x
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import time
from dataclasses import replace
from pathlib import Path

import torch
import torch.distributed as dist

from ..models.llama import PRESETS, LlamaConfig
from ..models.train import TrainConfig, Trainer, synthetic_batch
from ..utils.results import ROOT
from .traces import breakdown


def model_flops_per_token(cfg: LlamaConfig, seq: int) -> float:
    """Forward + backward FLOPs per trained token: 6 x (matrix parameters touched per token) plus causal
    attention (QK^T and PV, half the S x S square on average): 6 x layers x heads x head_dim x seq."""
    D = cfg.head_dim
    dense = cfg.layers * (cfg.hidden * (cfg.heads + 2 * cfg.kv_heads) * D + cfg.heads * D * cfg.hidden
                          + 3 * cfg.hidden * cfg.inter) + cfg.vocab * cfg.hidden
    return 6.0 * dense + 6.0 * cfg.layers * cfg.heads * D * seq


def measured_bf16_tflops() -> float | None:
    p = ROOT / "MEASURED_PEAKS.json"
    if not p.exists():
        return None
    d = json.loads(p.read_text())
    return d.get("bf16_tflops_sustained") or d.get("bf16_tflops")


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="1b", help="preset name (1b, 8b, 70b, tiny)")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (shorter runs)")
    ap.add_argument("--tp", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--global-seqs", type=int, default=8, help="sequences per step over all data-parallel ranks")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--profile", type=int, default=5)
    ap.add_argument("--remat", type=int, choices=[0, 1], default=0)
    ap.add_argument("--loss-parallel", type=int, choices=[0, 1], default=1)
    ap.add_argument("--out-dir", default=None)
    ap.add_argument("--device", default="auto", choices=["auto", "cuda", "cpu"])
    return ap.parse_args(argv)


def run(a, rank: int, world: int, device: torch.device) -> dict | None:
    """The measurement on an initialised process group (or world 1). Returns rank 0's summary."""
    cfg = PRESETS[a.model] if a.layers is None else replace(PRESETS[a.model], layers=a.layers)
    tr = Trainer(cfg, TrainConfig(tp=a.tp, remat=bool(a.remat), loss_parallel=bool(a.loss_parallel),
                                  bf16=device.type == "cuda"), device)
    assert a.global_seqs % tr.dp == 0, f"{a.global_seqs} sequences do not split over {tr.dp} data-parallel ranks"
    B = a.global_seqs // tr.dp
    cuda = device.type == "cuda"
    out = Path(a.out_dir or ROOT / "results" / "train_share" / time.strftime("%Y%m%d_%H%M%S"))
    out.mkdir(parents=True, exist_ok=True)
    step_no = [0]
    losses = []

    def one_step():
        host = synthetic_batch(cfg, B, a.seq, step_no[0], tr.dp_rank, pin=cuda)
        t = host.to(device, non_blocking=True)
        loss = tr.step(t[:, :-1], t[:, 1:])
        loss = loss.full_tensor() if hasattr(loss, "full_tensor") else loss
        losses.append(float(loss))  # the logger's read-back (host sync, as every step of a real run)
        step_no[0] += 1

    for _ in range(a.warmup):
        one_step()
    if world > 1:
        dist.barrier()
    if cuda:
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
        for s, e in ev:
            s.record()
            one_step()
            e.record()
        torch.cuda.synchronize()
        total_ms = sum(s.elapsed_time(e) for s, e in ev)
    else:
        t0 = time.perf_counter()
        for _ in range(a.steps):
            one_step()
        total_ms = 1e3 * (time.perf_counter() - t0)
    tot = torch.tensor([total_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    step_ms = float(tot) / max(1, a.steps)

    acts = [torch.profiler.ProfilerActivity.CPU] + ([torch.profiler.ProfilerActivity.CUDA] if cuda else [])
    with torch.profiler.profile(activities=acts) as prof:
        for _ in range(a.profile):
            with torch.profiler.record_function("train_step"):
                one_step()
    if cuda:
        torch.cuda.synchronize()
    prof.export_chrome_trace(str(out / f"trace_rank{rank}.json.gz"))
    if world > 1:
        dist.barrier()
    if rank != 0:
        return None
    tokens = a.global_seqs * a.seq
    flops = model_flops_per_token(cfg, a.seq) * tokens / (step_ms * 1e-3)
    peak = measured_bf16_tflops()
    summary = dict(model=cfg.name, layers=cfg.layers, world=world, tp=tr.tp, dp=tr.dp, seq=a.seq,
                   global_seqs=a.global_seqs, tokens_per_step=tokens, step_ms=step_ms,
                   tokens_per_s=tokens / (step_ms * 1e-3), tflops_per_gpu=flops / world / 1e12,
                   mfu_of_measured=(flops / world / 1e12 / peak) if (peak and cuda) else None,
                   loss_first=losses[0], loss_last=losses[-1], tokens_seen=tr.tokens_seen, remat=bool(a.remat),
                   device=device.type,
                   peak_mem_gb=(torch.cuda.max_memory_allocated(device) / 2**30) if cuda else None,
                   data="synthetic (random token ids, random init)")
    if a.profile > 0:
        summary["breakdown"] = breakdown(sorted(out.glob("trace_rank*.json.gz")), "train_step", step_us=step_ms * 1e3)
    (out / "summary.json").write_text(json.dumps(summary, indent=1))
    return summary


def main(argv=None):
    a = parse(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = a.device == "cuda" or (a.device == "auto" and torch.cuda.is_available())
    device = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if use_cuda:
        torch.cuda.set_device(device)
    if world > 1:
        kw = dict(device_id=device) if use_cuda else {}
        dist.init_process_group("nccl" if use_cuda else "gloo", timeout=datetime.timedelta(seconds=600), **kw)
    rank = dist.get_rank() if world > 1 else 0
    try:
        s = run(a, rank, world, device)
        if s is not None:
            print(json.dumps({k: v for k, v in s.items() if k != "breakdown"} |
                             {"breakdown": {k: v for k, v in s.get("breakdown", {}).items() if k != "raw"}}), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
