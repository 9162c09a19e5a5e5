"""Communication share of a decode or training step from profiler (Kineto/Chrome) traces.

Capability of the reference's exp/M5_e2e_comm_share/traces.py:87-167: split each step's GPU time into
compute-only, exposed communication (comm kernels not overlapped by compute), overlap and idle, and
split exposed communication into transfer and waiting using the shortest duration of the same
collective across ranks (the last rank to arrive barely waits). Communication kernels are matched
by name; here they are this library's fused collectives and NCCL's kernels.

    python -m comm_opt_b200.harness.traces trace_rank*.json --step-re "decode_step"
    python -m comm_opt_b200.harness.traces trace_rank*.json --step-re train_step --breakdown --step-us 700000

`breakdown` adds the reference's training analysis (exp/M5_e2e_comm_share/analyze_train.py:38-83 with
traces.py:143-167): exposed time per collective type and the compute slowdown caused by overlap.
"""
from __future__ import annotations

import argparse
import gzip
import json
import re
import statistics
from pathlib import Path

COMM_RE = re.compile(r"k_oneshot|k_twoshot|k_allgather|nccl|cross_device_reduce|custom_?all_?reduce|allreduce_fusion|"
                     r"one_shot_all_reduce|two_shot_all_reduce|multimem", re.I)
# kernels that do a GEMM and the collective together (layer-boundary fusion): counted as compute in the
# split above, and reported on their own as fused_us
FUSED_RE = re.compile(r"k_gemm_push|k_ar_norm_gemm", re.I)
GPU_CATS = {"kernel", "gpu_memcpy", "gpu_memset"}


def union(iv: list[tuple[float, float]]) -> list[tuple[float, float]]:
    out: list[list[float]] = []
    for s, e in sorted(iv):
        if out and s <= out[-1][1]:
            out[-1][1] = max(out[-1][1], e)
        else:
            out.append([s, e])
    return [(a, b) for a, b in out]


def length(iv) -> float:
    return sum(e - s for s, e in iv)


def intersect(a, b) -> list[tuple[float, float]]:
    out, i, j = [], 0, 0
    while i < len(a) and j < len(b):
        s, e = max(a[i][0], b[j][0]), min(a[i][1], b[j][1])
        if s < e:
            out.append((s, e))
        if a[i][1] < b[j][1]:
            i += 1
        else:
            j += 1
    return out


def clip(iv, s: float, e: float):
    return [(max(a, s), min(b, e)) for a, b in iv if b > s and a < e]


def load_events(path: Path) -> list[dict]:
    opener = gzip.open if str(path).endswith(".gz") else open
    with opener(path, "rt") as f:
        return json.load(f)["traceEvents"]


def step_marks(events: list[dict], step_re: str) -> list[tuple[float, float]]:
    """Step spans from annotations matching step_re: the GPU-side copies (the span of the step's kernels)
    when the trace has them, else the CPU-side ones. A record_function range appears once on each side."""
    out = {}
    for e in events:
        if e.get("cat") in ("gpu_user_annotation", "user_annotation") and re.search(step_re, e.get("name", "")):
            out.setdefault(e["cat"], []).append((e["ts"], e["ts"] + e.get("dur", 0)))
    return sorted(out.get("gpu_user_annotation") or out.get("user_annotation") or [])


def decompose_rank(events: list[dict], step_re: str) -> tuple[list[dict], list[float]]:
    """Per step (between consecutive step annotations): compute-only, exposed comm, overlap, idle (us);
    also the durations of the comm kernels in order (for the cross-rank transfer estimate)."""
    work = [e for e in events if e.get("cat") in GPU_CATS and e.get("dur", 0) > 0]
    comm = union([(e["ts"], e["ts"] + e["dur"]) for e in work if COMM_RE.search(e.get("name", ""))])
    comp = union([(e["ts"], e["ts"] + e["dur"]) for e in work if not COMM_RE.search(e.get("name", ""))])
    fused = union([(e["ts"], e["ts"] + e["dur"]) for e in work if FUSED_RE.search(e.get("name", ""))])
    marks = step_marks(events, step_re)
    steps = []
    for s, e in marks:
        c, k = union(clip(comm, s, e)), union(clip(comp, s, e))
        both = intersect(c, k)
        busy = length(union(c + k))
        steps.append(dict(wall_us=e - s, compute_only_us=length(k) - length(both),
                          exposed_comm_us=length(c) - length(both), overlap_us=length(both), idle_us=e - s - busy,
                          comm_total_us=length(c), fused_us=length(union(clip(fused, s, e)))))
    comm_durs = [e["dur"] for e in sorted(work, key=lambda x: x["ts"]) if COMM_RE.search(e.get("name", ""))]
    return steps, comm_durs


def decompose(trace_files: list[Path], step_re: str) -> list[dict]:
    ranks = [decompose_rank(load_events(Path(f)), step_re) for f in trace_files]
    counts = {len(d) for _, d in ranks}
    transfer_frac = None
    if len(counts) == 1 and counts != {0} and len(ranks) > 1:
        n = counts.pop()
        mins = [min(d[i] for _, d in ranks) for i in range(n)]
        transfer_frac = [sum(mins) / max(1e-9, sum(d)) for _, d in ranks]
    rows = []
    for r, (steps, _) in enumerate(ranks):
        for i, st in enumerate(steps):
            frac = transfer_frac[r] if transfer_frac else 1.0
            rows.append(dict(rank=r, step=i, exposed_transfer_us=st["exposed_comm_us"] * frac,
                             exposed_wait_us=st["exposed_comm_us"] * (1 - frac), **st))
    return rows


_NCCL_ALGO_WORDS = {"RING", "TREE", "NVLS", "NVLSTREE", "COLLNET", "DIRECT", "CHAIN", "PAT", "LL", "LL128", "SIMPLE"}


def comm_type(name: str) -> str:
    """Collective type of a communication kernel: NCCL kernels by their collective, reduction and data type
    (ncclDevKernel_ReduceScatter_Sum_bf16_RING_LL -> ReduceScatter_Sum_bf16), others by function name."""
    n = re.sub(r"^(void )?", "", name)
    m = re.match(r"nccl(?:Dev)?Kernel_(.*)", n)
    if m:  # drop the algorithm / protocol words wherever the NCCL version puts them
        words = m.group(1).split("(")[0].split("_")
        return "_".join(w for w in words if w not in _NCCL_ALGO_WORDS)
    return re.split(r"[<(]", n)[0].strip()


def _window_kernels(events, window):
    s0, s1 = window
    return [e for e in events if e.get("cat") in GPU_CATS and e.get("dur", 0) > 0 and s0 <= e["ts"] < s1]


def exposed_by_type(events: list[dict], window: tuple[float, float]) -> dict[str, float]:
    """Exposed (not overlapped by any compute kernel) time of each communication kernel inside the window,
    summed per collective type (us)."""
    k = _window_kernels(events, window)
    comp = union([(e["ts"], e["ts"] + e["dur"]) for e in k if not COMM_RE.search(e.get("name", ""))])
    out: dict[str, float] = {}
    for e in k:
        if e.get("cat") != "kernel" or not COMM_RE.search(e.get("name", "")):
            continue
        iv = [(e["ts"], e["ts"] + e["dur"])]
        t = comm_type(e["name"])
        out[t] = out.get(t, 0.0) + e["dur"] - length(intersect(iv, comp))
    return out


def overlap_slowdown(events: list[dict], window: tuple[float, float], min_alone: int = 5) -> dict:
    """Hidden cost of overlapping communication with compute (the measure of Lee et al., arXiv 2507.03114):
    every compute kernel that spends more than half its time under a communication kernel is compared
    with the median duration of the same kernel (name and grid) when it ran with no communication; the
    sum of the excess is the extra time that overlap cost. Kernels seen alone fewer than min_alone times
    are left out (no stable baseline)."""
    k = [e for e in _window_kernels(events, window) if e.get("cat") == "kernel"]
    comm = union([(e["ts"], e["ts"] + e["dur"]) for e in k if COMM_RE.search(e.get("name", ""))])
    alone: dict[tuple, list[float]] = {}
    over: list[tuple[tuple, float]] = []
    for e in k:
        if COMM_RE.search(e.get("name", "")):
            continue
        key = (e["name"][:160], str(e.get("args", {}).get("grid")))
        ov = length(intersect([(e["ts"], e["ts"] + e["dur"])], comm)) > 0.5 * e["dur"] if comm else False
        if ov:
            over.append((key, e["dur"]))
        else:
            alone.setdefault(key, []).append(e["dur"])
    med = {key: statistics.median(v) for key, v in alone.items() if len(v) >= min_alone}
    matched = [(key, d) for key, d in over if key in med]
    return dict(extra_us=sum(d - med[key] for key, d in matched), overlapped_compute_us=sum(d for _, d in over),
                matched_overlapped_us=sum(d for _, d in matched))


def summarize(rows: list[dict]) -> dict:
    """Shares of the captured steps: per rank the ratio of sums (so compute-only + exposed + overlap + idle
    = 100 % on every rank), then the mean across ranks (which keeps that sum)."""
    parts = ("compute_only_us", "exposed_comm_us", "exposed_transfer_us", "exposed_wait_us", "overlap_us", "idle_us",
             "comm_total_us")
    ranks = sorted({r["rank"] for r in rows})
    out = {}
    for p in parts:
        fr = []
        for rk in ranks:
            mine = [r for r in rows if r["rank"] == rk]
            fr.append(sum(r[p] for r in mine) / max(1e-9, sum(r["wall_us"] for r in mine)))
        out[p.replace("_us", "_pct")] = 100 * sum(fr) / max(1, len(fr))
    walls = sorted(r["wall_us"] for r in rows)
    out["step_wall_us"] = walls[len(walls) // 2] if walls else 0.0
    out["n_steps"] = min((sum(1 for r in rows if r["rank"] == rk) for rk in ranks), default=0)
    return out


def breakdown(trace_files: list[Path], step_re: str, step_us: float | None = None) -> dict:
    """Where a step's time goes, as shares of the step time: compute (minus what overlap cost it), the hidden
    cost of overlap, exposed transfer, everything else (CPU overhead, waiting for other ranks, idle), the
    total communication cost (transfer + hidden cost) and the exposed time per collective type.
    step_us: the step time measured without the profiler (default: the profiled median)."""
    rows = decompose(trace_files, step_re)
    s = summarize(rows)
    t = step_us or s["step_wall_us"]
    ranks = sorted({r["rank"] for r in rows})

    def per_rank_mean(key):
        vals = [sum(r[key] for r in rows if r["rank"] == rk) / max(1, sum(1 for r in rows if r["rank"] == rk))
                for rk in ranks]
        return sum(vals) / max(1, len(vals))

    compute = per_rank_mean("compute_only_us") + per_rank_mean("overlap_us")
    transfer = per_rank_mean("exposed_transfer_us")
    hidden, by_type = [], {}
    for f in trace_files:
        ev = load_events(Path(f))
        marks = step_marks(ev, step_re)
        if not marks:
            continue
        window, n = (marks[0][0], marks[-1][1]), len(marks)
        for k, v in exposed_by_type(ev, window).items():
            by_type[k] = by_type.get(k, 0.0) + v / n / len(trace_files)
        hidden.append(overlap_slowdown(ev, window)["extra_us"] / n)
    hid = sum(hidden) / max(1, len(hidden))
    out = dict(step_us=t, profiled_step_us=s["step_wall_us"], n_steps=s["n_steps"],
               compute_pct=100 * (compute - hid) / t, hidden_cost_pct=100 * hid / t, transfer_pct=100 * transfer / t,
               other_pct=100 * (1 - (compute + transfer) / t), comm_cost_pct=100 * (transfer + hid) / t,
               raw=s)
    out.update({f"exposed_{k}_pct": 100 * v / t for k, v in sorted(by_type.items())})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("traces", nargs="+")
    ap.add_argument("--step-re", default="decode_step")
    ap.add_argument("--breakdown", action="store_true", help="shares of the step incl. hidden cost and per-type comm")
    ap.add_argument("--step-us", type=float, default=None, help="unprofiled step time for --breakdown")
    a = ap.parse_args()
    if a.breakdown:
        print(json.dumps(breakdown([Path(t) for t in a.traces], a.step_re, a.step_us), indent=1))
        return
    rows = decompose([Path(t) for t in a.traces], a.step_re)
    for r in rows:
        share = r["exposed_comm_us"] / r["wall_us"] if r["wall_us"] else 0.0
        print(f"rank {r['rank']} step {r['step']}: wall {r['wall_us']:.1f} us  compute-only {r['compute_only_us']:.1f}  "
              f"exposed comm {r['exposed_comm_us']:.1f} ({share * 100:.1f}%)  overlap {r['overlap_us']:.1f}  "
              f"idle {r['idle_us']:.1f}")


if __name__ == "__main__":
    main()
