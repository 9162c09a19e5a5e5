"""Summarise an ncu launch list (gpu__time_duration.sum per kernel, CSV) into per-kernel shares.

    python -m comm_opt_b200.harness.launch_table launches.csv --steps 3
"""
from __future__ import annotations

import argparse
import collections
import csv
import re


def load(path: str) -> list[dict]:
    rows, hdr = [], None
    for r in csv.reader(open(path)):
        if r and r[0] == "ID":
            hdr = r
            continue
        if hdr and len(r) == len(hdr):
            rows.append(dict(zip(hdr, r)))
    return rows


def short(name: str) -> str:
    name = re.sub(r"\(anonymous namespace\)::|cob::|unnamed>::", "", name)
    return name.split("(")[0][:70]


def summarize(rows: list[dict], steps: int = 1) -> list[tuple]:
    scale = {"nsecond": 1e-3, "ns": 1e-3, "usecond": 1.0, "us": 1.0, "msecond": 1e3, "ms": 1e3}
    agg = collections.defaultdict(lambda: [0, 0.0])
    for d in rows:
        if d.get("Metric Name") != "gpu__time_duration.sum":
            continue
        us = float(d["Metric Value"].replace(",", "")) * scale.get(d["Metric Unit"], 1.0)
        k = short(d["Kernel Name"])
        agg[k][0] += 1
        agg[k][1] += us
    tot = sum(v[1] for v in agg.values()) or 1.0
    return [(k, n // steps, us / steps, us / tot) for k, (n, us) in sorted(agg.items(), key=lambda kv: -kv[1][1])]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("csv")
    ap.add_argument("--steps", type=int, default=1)
    a = ap.parse_args()
    rows = summarize(load(a.csv), a.steps)
    print(f"{'share':>7s} {'us/step':>9s} {'n/step':>6s}  kernel")
    for k, n, us, frac in rows:
        print(f"{frac * 100:6.2f}% {us:9.1f} {n:6d}  {k}")
    print(f"total {sum(r[2] for r in rows):.1f} us/step")


if __name__ == "__main__":
    main()
