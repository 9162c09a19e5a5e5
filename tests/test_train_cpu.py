"""Training workload (TP x FSDP on a 2-D mesh) and the training comm-share analysis, on CPU / gloo ranks."""
import json
from dataclasses import replace

import torch

from conftest import run_gloo

from comm_opt_b200.models.llama import TINY

CFG = replace(TINY, hidden=128, layers=2, heads=8, kv_heads=4, head_dim=16, inter=256, vocab=512)
B, S, STEPS = 4, 16, 3


def _reference_losses(dp: int) -> list[float]:
    """One process, unsharded model, the concatenation of every data-parallel rank's batch."""
    from comm_opt_b200.models.train import TrainConfig, Trainer, synthetic_batch

    tr = Trainer(CFG, TrainConfig(tp=1, init="full", bf16=False, count_tokens=False), "cpu")
    out = []
    for st in range(STEPS):
        t = torch.cat([synthetic_batch(CFG, B // dp, S, st, r) for r in range(dp)])
        out.append(tr.step(t[:, :-1], t[:, 1:]).item())
    return out


def _sharded(rank, world, tp, remat, expected):
    import torch.distributed as dist

    from comm_opt_b200.models.train import TrainConfig, Trainer, synthetic_batch

    tr = Trainer(CFG, TrainConfig(tp=tp, init="full", bf16=False, remat=remat), "cpu")
    dp = world // tp
    assert (tr.tp, tr.dp) == (tp, dp)
    for st in range(STEPS):
        t = synthetic_batch(CFG, B // dp, S, st, tr.dp_rank)
        loss = tr.step(t[:, :-1], t[:, 1:])
        loss = loss.full_tensor() if hasattr(loss, "full_tensor") else loss
        ls = [torch.zeros(()) for _ in range(world)]
        dist.all_gather(ls, loss.reshape(()).contiguous())
        got = sum(ls[i * tp] for i in range(dp)).item() / dp  # mean over data-parallel groups
        assert abs(got - expected[st]) < 1e-4 * abs(expected[st]), (st, got, expected[st])
    # tensor-parallel shards: column-parallel weights split along rows, row-parallel along columns
    shapes = tr.local_shapes()
    if tp > 1 and dp == 1:
        assert shapes["layers.0.attention.wq.weight"] == (CFG.heads * CFG.head_dim // tp, CFG.hidden)
        assert shapes["layers.0.feed_forward.w2.weight"] == (CFG.hidden, CFG.inter // tp)


def test_train_tp2_matches_single_process():
    """Sequence-parallel TP=2: three AdamW steps (with gradient clipping) equal the unsharded model's."""
    run_gloo(_sharded, 2, 2, False, _reference_losses(1), timeout=300)


def test_train_tp2_fsdp2_with_remat_matches_single_process():
    """TP=2 x FSDP=2 on a 2-D mesh, activation checkpointing on: the mean loss over data-parallel groups
    equals the unsharded model trained on the concatenated batch."""
    run_gloo(_sharded, 4, 2, True, _reference_losses(2), timeout=300)


def _share(rank, world, out_dir):
    from comm_opt_b200.harness.train_share import parse, run

    a = parse(["--model", "tiny", "--layers", "1", "--tp", "2", "--seq", "32", "--global-seqs", "2", "--warmup", "1",
               "--steps", "1", "--profile", "1", "--out-dir", out_dir])
    s = run(a, rank, world, torch.device("cpu"))
    if rank == 0:
        assert s["tp"] == 2 and s["dp"] == 1 and s["step_ms"] > 0 and s["tokens_per_step"] == 64
        assert s["breakdown"]["n_steps"] == 1 and torch.isfinite(torch.tensor(s["loss_last"]))
        assert s["tokens_seen"] == 3 * 2 * 32  # warm-up + timed + profiled steps x 2 sequences x 32 tokens


def test_train_share_driver_gloo(tmp_path):
    run_gloo(_share, 2, str(tmp_path), timeout=300)
    assert sorted(p.name for p in tmp_path.glob("trace_rank*.json.gz")) == ["trace_rank0.json.gz", "trace_rank1.json.gz"]
    s = json.loads((tmp_path / "summary.json").read_text())
    assert {"compute_pct", "transfer_pct", "hidden_cost_pct", "other_pct"} <= set(s["breakdown"])


def test_training_breakdown_synthetic(tmp_path):
    """Exposed time per collective type, overlap slowdown and the step shares on a synthetic trace: one step
    of 100 us with a GEMM that runs 10 us alone (5 times) and 14 us under an all-gather."""
    from comm_opt_b200.harness.traces import breakdown, comm_type, exposed_by_type, overlap_slowdown, step_marks

    ev = [dict(cat="user_annotation", name="train_step", ts=0, dur=110),
          dict(cat="gpu_user_annotation", name="train_step", ts=0, dur=100)]
    t = 0
    for _ in range(5):
        ev.append(dict(cat="kernel", name="sm100_gemm", ts=t, dur=10, args=dict(grid=[148, 1, 1])))
        t += 10
    ev.append(dict(cat="kernel", name="ncclDevKernel_AllGather_RING_LL(x)", ts=50, dur=20))
    ev.append(dict(cat="kernel", name="sm100_gemm", ts=52, dur=14, args=dict(grid=[148, 1, 1])))
    ev.append(dict(cat="kernel", name="ncclDevKernel_ReduceScatter_Sum_float_RING_LL(x)", ts=80, dur=10))
    (tmp_path / "trace_rank0.json").write_text(json.dumps(dict(traceEvents=ev)))
    assert step_marks(ev, "train_step") == [(0, 100)]  # the GPU-side span, not both copies
    assert comm_type(ev[-1]["name"]) == "ReduceScatter_Sum_float"
    ex = exposed_by_type(ev, (0, 100))
    assert ex == {"AllGather": 6.0, "ReduceScatter_Sum_float": 10.0}
    sl = overlap_slowdown(ev, (0, 100))
    assert abs(sl["extra_us"] - 4.0) < 1e-9 and sl["overlapped_compute_us"] == 14
    b = breakdown([tmp_path / "trace_rank0.json"], "train_step", step_us=100.0)
    # compute kernels busy 64 us (50 alone + 14 overlapped), 4 us of it the overlap's cost; exposed comm 16 us
    assert abs(b["compute_pct"] - 60.0) < 1e-9 and abs(b["hidden_cost_pct"] - 4.0) < 1e-9
    assert abs(b["transfer_pct"] - 16.0) < 1e-9 and abs(b["other_pct"] - 20.0) < 1e-9
    assert abs(b["exposed_AllGather_pct"] - 6.0) < 1e-9
