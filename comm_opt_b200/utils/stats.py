"""Statistics helpers used by the sweeps and analyzers."""
from __future__ import annotations

import math


def percentile(xs, q: float) -> float:
    xs = sorted(xs)
    if not xs:
        return float("nan")
    k = (len(xs) - 1) * q
    f, c = math.floor(k), math.ceil(k)
    return xs[f] if f == c else xs[f] + (xs[c] - xs[f]) * (k - f)


def summary(xs) -> dict:
    xs = list(xs)
    return dict(n=len(xs), p50=percentile(xs, 0.5), p99=percentile(xs, 0.99), mean=sum(xs) / max(1, len(xs)),
                min=min(xs) if xs else float("nan"), max=max(xs) if xs else float("nan"))


def median_minmax(xs) -> dict:
    """Median and [min, max] over independent launches (the reference's reporting rule)."""
    return dict(med=percentile(xs, 0.5), lo=min(xs), hi=max(xs), n=len(xs))


def disjoint(a: dict, b: dict) -> bool:
    """[min, max] intervals do not overlap."""
    return a["hi"] < b["lo"] or b["hi"] < a["lo"]
