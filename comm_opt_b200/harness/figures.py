"""Figures and CSV tables from committed runs, written to figures/<exp>/<timestamp>/ (the reference's
analysis outputs, figures/<ID>/<ts>/*.csv and *.png, e.g. exp/M5_e2e_comm_share/analyze_train.py:86-124).
Plots are plain SVG written here (no plotting library in this stack):

  * fused-op sweep (sweep.json): p50 latency against message size per implementation, log-log;
  * layer-boundary bench (boundary.json): p50 per batch size per implementation, plus the roofline;
  * training / decode comm share (summary.json of harness/train_share.py): one stacked bar of the step.

    python -m comm_opt_b200.harness.figures results/fused_sweep/<ts> results/boundary_bench/<ts> ...
"""
from __future__ import annotations

import argparse
import csv
import json
import math
from pathlib import Path

from ..utils.results import ROOT

PALETTE = ("#2a78d6", "#eb6834", "#1baf7a", "#c43c8c", "#7a5af5", "#b38b00", "#52514e", "#00a3b4", "#d62a2a",
           "#898781")
W, H, ML, MR, MT, MB = 760, 430, 70, 190, 40, 55  # canvas and margins


def _esc(s: str) -> str:
    return str(s).replace("&", "&amp;").replace("<", "&lt;").replace(">", "&gt;")


def _ticks(lo: float, hi: float, log: bool) -> list[float]:
    if log:
        a, b = math.floor(math.log10(lo)), math.ceil(math.log10(hi))
        mult = (1, 2, 5) if b - a <= 3 else (1,)
        return [m * 10.0 ** e for e in range(a, b + 1) for m in mult]
    step = 10 ** math.floor(math.log10(max(hi - lo, 1e-12)))
    while (hi - lo) / step > 8:
        step *= 2
    t = math.floor(lo / step) * step
    out = []
    while t <= hi + 1e-9:
        out.append(t)
        t += step
    return out


def line_chart(series: dict[str, list[tuple[float, float]]], title: str, xlabel: str, ylabel: str,
               logx: bool = True, logy: bool = True, xfmt=None) -> str:
    """SVG line chart of {name: [(x, y), ...]} with a legend on the right."""
    pts = [p for s in series.values() for p in s if p[1] is not None and p[1] > 0]
    if not pts:
        return ""
    xs, ys = [p[0] for p in pts], [p[1] for p in pts]
    x0, x1 = min(xs), max(xs)
    y0, y1 = (min(ys) / 1.3, max(ys) * 1.3) if logy else (0.0, max(ys) * 1.1)
    if x0 == x1:
        x0, x1 = x0 / 2, x1 * 2
    fx = (lambda v: math.log10(v)) if logx else (lambda v: v)
    fy = (lambda v: math.log10(v)) if logy else (lambda v: v)
    pw, ph = W - ML - MR, H - MT - MB

    def X(v):
        return ML + (fx(v) - fx(x0)) / (fx(x1) - fx(x0)) * pw

    def Y(v):
        return MT + ph - (fy(v) - fy(y0)) / (fy(y1) - fy(y0)) * ph

    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{H}" font-family="sans-serif" font-size="11">',
           f'<rect width="{W}" height="{H}" fill="#fcfcfb"/>',
           f'<text x="{ML}" y="22" font-size="13" fill="#0b0b0b">{_esc(title)}</text>']
    for t in _ticks(y0, y1, logy):
        if y0 <= t <= y1:
            out.append(f'<line x1="{ML}" x2="{ML + pw}" y1="{Y(t):.1f}" y2="{Y(t):.1f}" stroke="#e4e3df"/>')
            out.append(f'<text x="{ML - 6}" y="{Y(t) + 4:.1f}" text-anchor="end" fill="#52514e">{t:g}</text>')
    xt = sorted({p[0] for p in pts})
    if len(xt) > 12:
        xt = xt[:: math.ceil(len(xt) / 12)]
    for t in xt:
        out.append(f'<text x="{X(t):.1f}" y="{MT + ph + 16}" text-anchor="middle" fill="#52514e">'
                   f'{_esc(xfmt(t) if xfmt else f"{t:g}")}</text>')
    out.append(f'<line x1="{ML}" x2="{ML + pw}" y1="{MT + ph}" y2="{MT + ph}" stroke="#898781"/>')
    out.append(f'<text x="{ML + pw / 2}" y="{H - 12}" text-anchor="middle" fill="#52514e">{_esc(xlabel)}</text>')
    out.append(f'<text x="16" y="{MT + ph / 2}" transform="rotate(-90 16 {MT + ph / 2})" text-anchor="middle" '
               f'fill="#52514e">{_esc(ylabel)}</text>')
    for i, (name, s) in enumerate(series.items()):
        col = PALETTE[i % len(PALETTE)]
        good = [(x, y) for x, y in sorted(s) if y is not None and y > 0]
        if not good:
            continue
        d = " ".join(f"{'M' if j == 0 else 'L'}{X(x):.1f},{Y(y):.1f}" for j, (x, y) in enumerate(good))
        out.append(f'<path d="{d}" fill="none" stroke="{col}" stroke-width="1.8"/>')
        for x, y in good:
            out.append(f'<circle cx="{X(x):.1f}" cy="{Y(y):.1f}" r="2.5" fill="{col}"/>')
        ly = MT + 14 + 16 * i
        out.append(f'<line x1="{W - MR + 12}" x2="{W - MR + 30}" y1="{ly - 4}" y2="{ly - 4}" stroke="{col}" '
                   f'stroke-width="2"/><text x="{W - MR + 36}" y="{ly}" fill="#0b0b0b">{_esc(name)}</text>')
    out.append("</svg>")
    return "\n".join(out)


def stacked_bar(parts: list[tuple[str, float]], title: str) -> str:
    """One horizontal bar of percentages (negative parts drawn as 0)."""
    pw = W - 2 * ML
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="150" font-family="sans-serif" font-size="11">',
           f'<rect width="{W}" height="150" fill="#fcfcfb"/>',
           f'<text x="{ML}" y="22" font-size="13" fill="#0b0b0b">{_esc(title)}</text>']
    x = ML
    for i, (name, pct) in enumerate(parts):
        w = max(0.0, pct) / 100 * pw
        col = PALETTE[i % len(PALETTE)]
        out.append(f'<rect x="{x:.1f}" y="40" width="{w:.1f}" height="34" fill="{col}"/>')
        if w > 28:
            out.append(f'<text x="{x + w / 2:.1f}" y="61" text-anchor="middle" fill="#fcfcfb">{pct:.0f}%</text>')
        out.append(f'<rect x="{ML + 150 * (i % 4)}" y="{92 + 20 * (i // 4)}" width="10" height="10" fill="{col}"/>'
                   f'<text x="{ML + 150 * (i % 4) + 14}" y="{101 + 20 * (i // 4)}" fill="#0b0b0b">{_esc(name)}</text>')
        x += w
    out.append("</svg>")
    return "\n".join(out)


def _kb(v: float) -> str:
    return f"{v / 1024:g}K" if v < 1 << 20 else f"{v / (1 << 20):g}M"


def _write_csv(path: Path, rows: list[dict], cols: list[str]):
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=cols, extrasaction="ignore")
        w.writeheader()
        for r in rows:
            w.writerow(r)


def sweep_figures(doc: dict, out: Path, link_gbs: float | None = None) -> list[Path]:
    """Latency per message size, and the achieved fraction of the NVLink roofline at `link_gbs` (default:
    the newest committed platform record, utils.peaks.link_gbs)."""
    rows = [r for r in doc["rows"] if r.get("correct") and r.get("p50_us")]
    series: dict[str, list] = {}
    for r in rows:
        series.setdefault(r["impl"], []).append((r["bytes"], r["p50_us"]))
    _write_csv(out / "per_op.csv", doc["rows"], ["impl", "world", "dtype", "hidden", "tokens", "bytes", "p50_us",
                                                "p99_us", "mean_us", "max_rel_err", "correct", "skip", "error"])
    r0 = doc["rows"][0] if doc["rows"] else {}
    svg = line_chart(series, f"fused all-reduce + residual + RMSNorm, {doc.get('world')} GPUs, "
                             f"hidden {r0.get('hidden')} {r0.get('dtype')} (p50 per op, max over ranks)",
                     "message size (bytes)", "us", xfmt=_kb)
    (out / "latency.svg").write_text(svg)
    # achieved fraction of the NVLink roofline (analyze_sweep.roofline_table): ours and the best baseline
    from .analyze_sweep import roofline_table

    _, summ = roofline_table(doc["rows"], link_gbs)
    frac = {"best of ours": [(s["bytes"], s["fraction"]) for s in summ if s["fraction"]],
            "best baseline": [(s["bytes"], s["baseline_fraction"]) for s in summ if s["baseline_fraction"]]}
    w = doc.get("world") or 2
    gbs = summ[0]["link_gbs"] if summ else link_gbs
    _write_csv(out / "roofline.csv", summ, ["world", "tokens", "target_us", "ours", "fraction", "baseline",
                                            "baseline_fraction"])
    (out / "roofline.svg").write_text(line_chart(
        frac, f"fraction of the NVLink roofline (2 (W-1)/W x S at {gbs:.0f} GB/s measured), {w} GPUs",
        "message size (bytes)",
        "fraction", xfmt=_kb))
    return [out / "per_op.csv", out / "latency.svg", out / "roofline.csv", out / "roofline.svg"]


def boundary_figures(doc: dict, out: Path) -> list[Path]:
    rows = [r for r in doc["rows"] if r.get("correct") and not r.get("error") and r.get("p50_us")]
    series: dict[str, list] = {}
    for r in rows:
        series.setdefault(r["impl"], []).append((r["batch"], r["p50_us"]))
    roof = sorted({(r["batch"], r["roofline_us"]) for r in doc["rows"] if r.get("roofline_us")})
    if roof:
        series["roofline"] = roof
    _write_csv(out / "boundary.csv", doc["rows"], ["impl", "world", "batch", "p50_us", "p99_us", "max_rel_err",
                                                  "correct", "roofline_us", "frac_of_roofline", "error"])
    svg = line_chart(series, f"layer boundary GEMM -> all-reduce + RMSNorm -> GEMM, {doc.get('world')} GPUs (p50)",
                     "batch (tokens)", "us")
    (out / "boundary.svg").write_text(svg)
    return [out / "boundary.csv", out / "boundary.svg"]


def share_figures(doc: dict, out: Path) -> list[Path]:
    b = doc.get("breakdown", {})
    parts = [("compute", b.get("compute_pct", 0.0)), ("overlap cost", b.get("hidden_cost_pct", 0.0)),
             ("exposed transfer", b.get("transfer_pct", 0.0)), ("other (CPU, wait, idle)", b.get("other_pct", 0.0))]
    _write_csv(out / "share.csv", [dict(doc, **{k: v for k, v in b.items() if k != "raw"})],
               ["model", "world", "tp", "dp", "step_ms", "tokens_per_s", "compute_pct", "hidden_cost_pct",
                "transfer_pct", "other_pct", "comm_cost_pct"])
    title = (f"{doc.get('model')} TP={doc.get('tp')} x FSDP={doc.get('dp')}: {doc.get('step_ms', 0):.0f} ms/step")
    (out / "share.svg").write_text(stacked_bar(parts, title))
    return [out / "share.csv", out / "share.svg"]


def render(run_dir: Path, base: Path | None = None, link_gbs: float | None = None) -> list[Path]:
    """Figures of one run directory into <base>/figures/<exp>/<ts>/ (exp and ts from the run's path)."""
    run_dir = Path(run_dir)
    out = (base or ROOT) / "figures" / run_dir.parent.name / run_dir.name
    out.mkdir(parents=True, exist_ok=True)
    if (run_dir / "sweep.json").exists():
        return sweep_figures(json.loads((run_dir / "sweep.json").read_text()), out, link_gbs)
    for name, fn in (("boundary.json", boundary_figures), ("summary.json", share_figures)):
        if (run_dir / name).exists():
            return fn(json.loads((run_dir / name).read_text()), out)
    raise ValueError(f"no known result file in {run_dir}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("runs", nargs="+")
    a = ap.parse_args()
    for r in a.runs:
        for p in render(Path(r)):
            print(p)


if __name__ == "__main__":
    main()
