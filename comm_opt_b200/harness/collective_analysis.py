"""Loader and statistics for collective sweeps (the reference's exp/lib/nccljson.py:9-43 and the bound
of exp/M6_allreduce_bakeoff/analyze.py:106-116), for the JSON written by harness/collectives.py.

    python -m comm_opt_b200.harness.collective_analysis results/collective_baseline/<ts>/ --coll all_reduce
"""
from __future__ import annotations

import argparse
import csv
import json
import sys
from pathlib import Path

from ..utils.stats import disjoint, median_minmax  # noqa: F401  (re-exported for analyzers)


def load_run(run_dir: Path) -> list[dict]:
    """One row per (job, size) from every job JSON listed in schedule.tsv."""
    run_dir = Path(run_dir)
    rows = []
    sched = run_dir / "schedule.tsv"
    tags = []
    if sched.exists():
        for rec in csv.DictReader(open(sched), delimiter="\t"):
            tags.append((rec["tag"], int(rec["order"]), json.loads(rec["extra"]) if rec.get("extra") else {}))
    else:
        tags = [(p.stem, i, {}) for i, p in enumerate(sorted(run_dir.glob("*.json")))]
    for tag, order, extra in tags:
        f = run_dir / f"{tag}.json"
        try:
            doc = json.loads(f.read_text())
        except (OSError, json.JSONDecodeError) as e:
            print(f"skip {f.name}: {e}", file=sys.stderr)
            continue
        for r in doc["results"]:
            rows.append(dict(tag=tag, order=order, variant=extra.get("variant", "default"), **r))
    return rows


def summarize(rows: list[dict], keys: tuple, value: str = "busbw") -> dict:
    """Median and [min, max] across independent launches for every key tuple."""
    groups: dict[tuple, list] = {}
    for r in rows:
        groups.setdefault(tuple(r[k] for k in keys), []).append(r[value])
    return {k: median_minmax(v) for k, v in groups.items()}


def achievable_us(size_bytes: int, world: int, l0_us: float, bw_gbs: float) -> float:
    """Latency-bandwidth bound of an all-reduce: L0 + 2(n-1)/n * S / B (a reference point, not a law)."""
    return l0_us + 2 * (world - 1) / world * size_bytes / (bw_gbs * 1e3)


def fit_bound(rows: list[dict]) -> tuple[float, float]:
    """L0 = smallest-message latency, B = peak bus bandwidth of the all_reduce rows."""
    ar = [r for r in rows if r["coll"] == "all_reduce"]
    return min(r["p50_us"] for r in ar), max(r["busbw"] for r in ar)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("run_dir")
    ap.add_argument("--coll", default=None)
    a = ap.parse_args()
    rows = load_run(Path(a.run_dir))
    if a.coll:
        rows = [r for r in rows if r["coll"] == a.coll]
    s = summarize(rows, ("coll", "world", "variant", "size"), "p50_us")
    for k, v in sorted(s.items()):
        print(f"{k[0]:15s} w{k[1]} {k[2]:10s} {k[3]:>12d} B  p50 {v['med']:9.2f} us  [{v['lo']:.2f}, {v['hi']:.2f}] n={v['n']}")


if __name__ == "__main__":
    main()
