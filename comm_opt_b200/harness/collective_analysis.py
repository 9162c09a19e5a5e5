"""Loader and statistics for collective sweeps (the reference's exp/lib/nccljson.py:9-43 and the bound
of exp/M6_allreduce_bakeoff/analyze.py:106-116), for the JSON written by harness/collectives.py, with
NCCL's own set-up of each job read from its INIT / ENV / GRAPH log and the GPU-set comparison of the
repeat study (exp/M4_repeat).

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
        nccl = load_nccl_logs(run_dir, tag)
        for r in doc["results"]:
            rows.append(dict(tag=tag, order=order, variant=extra.get("variant", "default"),
                             gpuset=extra.get("gpuset", "A"), rep=extra.get("rep", 0), nccl=nccl, **r))
    return rows


_NCCL_PATTERNS = {
    "nccl_version": (r"NCCL version ([\w.+-]+)", str),
    "nranks": (r"nRanks (\d+)", int),
    "coll_channels": (r"(\d+) coll channels", int),
    "nvls_channels": (r"(\d+) nvls channels", int),
    "p2p_channels": (r"(\d+) p2p channels(?!\s*per)", int),
    "p2p_channels_per_peer": (r"(\d+) p2p channels per peer", int),
    "rings": (r"Channel (\d+)/\d+ :", lambda v: v),
}


def nccl_log_summary(text: str) -> dict:
    """What NCCL set up for a communicator, from its NCCL_DEBUG=INFO (INIT, ENV, GRAPH) log: version, ranks,
    collective / NVLS / P2P channel counts, number of ring channels, whether NVLS multicast was available,
    and the NCCL_* settings it reported. Fields it did not print stay absent."""
    import re

    out: dict = {}
    for key, (pat, conv) in _NCCL_PATTERNS.items():
        found = re.findall(pat, text)
        if not found:
            continue
        out[key] = len(set(found)) if key == "rings" else conv(found[0])
    if re.search(r"NVLS multicast support is available", text):
        out["nvls"] = True
    elif re.search(r"NVLS multicast support is not available|NVLS.*disabled", text, re.I):
        out["nvls"] = False
    env = dict(re.findall(r"(NCCL_[A-Z0-9_]+) set by environment to (\S+)", text))
    if env:
        out["env"] = env
    return out


def load_nccl_logs(run_dir: Path, tag: str) -> dict:
    """Summary of the first NCCL log file of a job (<tag>.nccl.<host>.<pid>.log, one per rank)."""
    logs = sorted(Path(run_dir).glob(f"{tag}.nccl.*.log"))
    return nccl_log_summary(logs[0].read_text(errors="replace")) if logs else {}


def compare_gpusets(rows: list[dict], value: str = "busbw", keys: tuple = ("coll", "world", "size")) -> list[dict]:
    """Per key: median [min, max] of set A and of set B over repeated launches, their relative difference
    and whether the intervals are disjoint (the reference's two-GPU-set rule, exp/M4_repeat/README.md)."""
    a = summarize([r for r in rows if r.get("gpuset", "A") == "A"], keys, value)
    b = summarize([r for r in rows if r.get("gpuset") == "B"], keys, value)
    out = []
    for k in sorted(set(a) & set(b)):
        out.append(dict(zip(keys, k), a=a[k], b=b[k], rel_diff=abs(a[k]["med"] - b[k]["med"]) / max(1e-12, a[k]["med"]),
                        disjoint=disjoint(a[k], b[k])))
    return out


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
    ap.add_argument("--gpusets", action="store_true", help="compare GPU sets A and B (repeat plan)")
    a = ap.parse_args()
    rows = load_run(Path(a.run_dir))
    if a.coll:
        rows = [r for r in rows if r["coll"] == a.coll]
    if a.gpusets:
        for c in compare_gpusets(rows):
            print(f"{c['coll']:15s} w{c['world']} {c['size']:>12d} B  A {c['a']['med']:8.1f} B {c['b']['med']:8.1f} GB/s "
                  f"diff {100 * c['rel_diff']:5.1f}%{'  disjoint' if c['disjoint'] else ''}")
        return
    s = summarize(rows, ("coll", "world", "variant", "size"), "p50_us")
    for k, v in sorted(s.items()):
        print(f"{k[0]:15s} w{k[1]} {k[2]:10s} {k[3]:>12d} B  p50 {v['med']:9.2f} us  [{v['lo']:.2f}, {v['hi']:.2f}] n={v['n']}")


if __name__ == "__main__":
    main()
