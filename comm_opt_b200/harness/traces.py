"""Communication share of a decode step from profiler (Kineto/Chrome) traces.

Capability of the reference's exp/M5_e2e_comm_share/traces.py:87-167: split each step's GPU time into
compute-only, exposed communication (comm kernels not overlapped by compute), overlap and idle, and
split exposed communication into transfer and waiting using the shortest duration of the same
collective across ranks (the last rank to arrive barely waits). Communication kernels are matched
by name; here they are this library's fused collectives and NCCL's kernels.

    python -m comm_opt_b200.harness.traces trace_rank*.json --step-re "decode_step"
"""
from __future__ import annotations

import argparse
import gzip
import json
import re
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


def decompose_rank(events: list[dict], step_re: str) -> tuple[list[dict], list[float]]:
    """Per step (between consecutive step annotations): compute-only, exposed comm, overlap, idle (us);
    also the durations of the comm kernels in order (for the cross-rank transfer estimate)."""
    work = [e for e in events if e.get("cat") in GPU_CATS and e.get("dur", 0) > 0]
    comm = union([(e["ts"], e["ts"] + e["dur"]) for e in work if COMM_RE.search(e.get("name", ""))])
    comp = union([(e["ts"], e["ts"] + e["dur"]) for e in work if not COMM_RE.search(e.get("name", ""))])
    fused = union([(e["ts"], e["ts"] + e["dur"]) for e in work if FUSED_RE.search(e.get("name", ""))])
    marks = sorted((e["ts"], e["ts"] + e.get("dur", 0)) for e in events
                   if e.get("cat") in ("gpu_user_annotation", "user_annotation") and re.search(step_re, e.get("name", "")))
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("traces", nargs="+")
    ap.add_argument("--step-re", default="decode_step")
    a = ap.parse_args()
    rows = decompose([Path(t) for t in a.traces], a.step_re)
    for r in rows:
        share = r["exposed_comm_us"] / r["wall_us"] if r["wall_us"] else 0.0
        print(f"rank {r['rank']} step {r['step']}: wall {r['wall_us']:.1f} us  compute-only {r['compute_only_us']:.1f}  "
              f"exposed comm {r['exposed_comm_us']:.1f} ({share * 100:.1f}%)  overlap {r['overlap_us']:.1f}  "
              f"idle {r['idle_us']:.1f}")


if __name__ == "__main__":
    main()
