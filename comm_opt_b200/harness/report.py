"""Markdown tables from committed runs: layer-boundary bench, all-reduce bake-off, phase profiles and
bench.py JSON lines (the fused-op sweep has its own analyzer, harness/analyze_sweep.py).

    python -m comm_opt_b200.harness.report results/boundary_bench/<ts> results/bench/bench_n8_fused.json ...
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path


def _fmt(v, nd=2):
    return "-" if v is None else (f"{v:.{nd}f}" if isinstance(v, float) else str(v))


def boundary_table(doc: dict) -> str:
    rows = doc["rows"]
    impls = list(dict.fromkeys(r["impl"] for r in rows))
    out = [f"layer boundary, world {doc['world']} (p50 us; roofline fraction of the fused path)", "",
           "| B | " + " | ".join(impls) + " | roofline us | fused / roofline |", "|" + "---|" * (len(impls) + 3)]
    for B in sorted({r["batch"] for r in rows}):
        cells = []
        roof, frac = None, None
        for i in impls:
            r = next((x for x in rows if x["batch"] == B and x["impl"] == i), None)
            ok = r and r.get("correct") and not r.get("error")
            cells.append(_fmt(r["p50_us"]) if ok else ("wrong" if r and not r.get("correct") else "-"))
            if r and i == "fused":
                roof, frac = r.get("roofline_us"), r.get("frac_of_roofline")
        out.append(f"| {B} | " + " | ".join(cells) + f" | {_fmt(roof)} | {_fmt(frac, 3)} |")
    return "\n".join(out)


def bakeoff_table(doc: dict) -> str:
    rows = doc["rows"]
    impls = list(dict.fromkeys(r["impl"] for r in rows))
    out = [f"all-reduce bake-off, world {doc['world']} (p50 us)", "",
           "| KB | " + " | ".join(impls) + " |", "|" + "---|" * (len(impls) + 1)]
    for nb in sorted({r["bytes"] for r in rows}):
        cells = []
        for i in impls:
            r = next((x for x in rows if x["bytes"] == nb and x["impl"] == i), None)
            cells.append(_fmt(r["p50_us"]) if r and r.get("correct") and r.get("p50_us") else
                         ("skip" if r and r.get("skip") else "-"))
        out.append(f"| {nb >> 10} | " + " | ".join(cells) + " |")
    return "\n".join(out)


def phases_table(doc: dict) -> str:
    keys = ("op_us", "op_us_stamped", "sent", "reduced", "received", "done", "gap")
    out = [f"phase profile, world {doc['world']} (us from the earliest block's start, max over ranks)", "",
           "| variant | tokens | " + " | ".join(keys) + " |", "|" + "---|" * (len(keys) + 2)]
    for r in doc["rows"]:
        out.append(f"| {r['variant']} | {r['tokens']} | " + " | ".join(_fmt(r.get(k)) for k in keys) + " |")
    return "\n".join(out)


def bench_table(lines: list[dict]) -> str:
    out = ["bench.py", "", "| metric | GPUs | ms/token | e2e ms/token | kernels/step | config |", "|---|---|---|---|---|---|"]
    for d in lines:
        if "unavailable" in d:
            out.append(f"| {d.get('impl')} | - | - | - | - | unavailable: {d['unavailable'][:60]} |")
            continue
        cfg = d.get("config", {})
        extra = ", ".join(f"{k}={cfg[k]}" for k in ("parallelism", "global_batch", "fuse_boundary", "collective",
                                                    "l2_prefetch_tiles") if cfg.get(k) not in (None, 0))
        fb = cfg.get("fused_boundaries")
        if fb:  # which boundary kinds the capture kept fused, and the step time of each choice
            kinds = "+".join(k for k in ("attention_out", "mlp_out") if fb.get(k)) or "none"
            times = fb.get("step_ms_by_choice") or {}
            extra += f", fused={kinds}" + (" (" + " ".join(f"{k}:{v:.3f}" for k, v in sorted(times.items())) + ")"
                                           if times else "")
        out.append(f"| {d['metric']} | {d['n_gpus']} | {_fmt(d['value'], 3)} | {_fmt(d.get('e2e', {}).get('value'), 3)} "
                   f"| {d.get('kernels_per_step', '-')} | {extra} |")
    return "\n".join(out)


def render(path: Path) -> str:
    path = Path(path)
    if path.is_dir():
        for name, fn in (("boundary.json", boundary_table), ("bakeoff.json", bakeoff_table),
                         ("phases.json", phases_table)):
            if (path / name).exists():
                return fn(json.loads((path / name).read_text()))
        raise ValueError(f"no known result file in {path}")
    lines = [json.loads(l) for l in path.read_text().splitlines() if l.strip().startswith("{")]
    return bench_table(lines)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("paths", nargs="+")
    a = ap.parse_args()
    print("\n\n".join(render(Path(p)) for p in a.paths))


if __name__ == "__main__":
    main()
