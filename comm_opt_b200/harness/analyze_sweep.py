"""Analyzer of fused-op sweeps: per-size table of p50 device latency for every implementation, the
speedup of our best measured variant over the best baseline, and (``--calibrate``) the measured
variant table used by ``TPCommunicator`` (the reference's calibrate step, exp/M18_incremental/run_b.py:60-73).

    python -m comm_opt_b200.harness.analyze_sweep results/fused_sweep/<ts>/sweep.json [--calibrate]
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

from ..parallel.variant_table import VARIANTS, Choice, VariantTable

BASELINES = ("nccl_norm", "vllm_car", "trt_oneshot", "trt_twoshot", "ref_m16nf")


def load(paths: list[str]) -> list[dict]:
    rows = []
    for p in paths:
        d = json.loads(Path(p).read_text())
        rows += d["rows"]
    return rows


def table(rows: list[dict]) -> tuple[str, list[dict]]:
    impls = sorted({r["impl"] for r in rows}, key=lambda s: (not s.startswith("ours"), s))
    out, summary = [], []
    for world in sorted({r["world"] for r in rows}):
        sub = [r for r in rows if r["world"] == world]
        sizes = sorted({r["tokens"] for r in sub})
        out.append(f"\n## world {world}, hidden {sub[0]['hidden']}, {sub[0]['dtype']}: p50 us per op (max over ranks)\n")
        out.append("| tokens | KB | " + " | ".join(impls) + " | best ours | best baseline | speedup |")
        out.append("|" + "---|" * (len(impls) + 5))
        for T in sizes:
            cells, best_o, best_b = [], (None, 1e30), (None, 1e30)
            for name in impls:
                r = next((x for x in sub if x["tokens"] == T and x["impl"] == name), None)
                v = r and r["p50_us"] if r and r["correct"] else None
                cells.append(f"{v:.2f}" if v else ("skip" if r and r["skip"] else "-"))
                if v and name.startswith("ours") and name != "ours:auto" and v < best_o[1]:
                    best_o = (name, v)
                if v and name in BASELINES and v < best_b[1]:
                    best_b = (name, v)
            kb = T * sub[0]["hidden"] * 2 // 1024
            sp = best_b[1] / best_o[1] if best_o[0] and best_b[0] else None
            out.append(f"| {T} | {kb} | " + " | ".join(cells) +
                       f" | {best_o[0] or '-'} | {best_b[0] or '-'} | {sp:.2f}x |" if sp else
                       f"| {T} | {kb} | " + " | ".join(cells) + " | - | - | - |")
            summary.append(dict(world=world, tokens=T, kb=kb, best_ours=best_o, best_baseline=best_b, speedup=sp))
    return "\n".join(out), summary


def repeats(rows: list[dict], ours: str, base: str) -> list[dict]:
    """Independent launches of the same configuration (several sweeps): per (world, tokens) the median
    and [min, max] of the per-launch p50 for `ours` and `base`, and whether the difference is
    "effective" by the reference's rule (>= 3 % and disjoint [min, max] intervals,
    exp/M18_incremental/README.md:34-40)."""
    from ..utils.stats import disjoint, median_minmax

    out = []
    keys = sorted({(r["world"], r["tokens"]) for r in rows})
    for w, T in keys:
        a = [r["p50_us"] for r in rows if (r["world"], r["tokens"], r["impl"]) == (w, T, ours) and r["correct"]
             and r["p50_us"]]
        b = [r["p50_us"] for r in rows if (r["world"], r["tokens"], r["impl"]) == (w, T, base) and r["correct"]
             and r["p50_us"]]
        if not a or not b:
            continue
        ma, mb = median_minmax(a), median_minmax(b)
        gain = mb["med"] / ma["med"] - 1.0
        out.append(dict(world=w, tokens=T, ours=ma, base=mb, gain=gain,
                        effective=abs(gain) >= 0.03 and disjoint(ma, mb) and len(a) >= 3 and len(b) >= 3))
    return out


def expected_tx_bytes(impl: str, msg: int, world: int) -> float | None:
    """Bytes one rank sends over NVLink per call, by algorithm (flags and row sums left out):
    one-shot push or pull, (W - 1) S (every peer gets, or reads, the whole message); two-shot
    reduce-scatter + all-gather, 2 (W - 1) / W S; NVSwitch multicast one-shot, W S (every rank's
    ld_reduce reads every GPU's copy through the switch); multicast two-shot, S + S / W (each slice read
    once, the reduced slice stored once for the switch to replicate). None for an unknown algorithm
    (NCCL picks its own)."""
    name = impl.split(":", 1)[-1]
    one, two = (world - 1) * msg, 2 * (world - 1) / world * msg
    return {"lamport_1s": one, "lamport_1sx": one, "pull_1s": one, "trt_oneshot": one, "lamport_2s": two, "pull_2s": two,
            "trt_twoshot": two, "ref_m16nf": two, "nvls_1s": world * msg, "nvls_2s": msg + msg / world}.get(name)


def link_table(rows: list[dict]) -> str:
    """Measured NVLink bytes sent per call (max over ranks, NVML counters) against the algorithm's bytes."""
    out = ["| impl | world | tokens | KB | measured tx KB/op | expected KB/op | ratio |", "|---|---|---|---|---|---|---|"]
    for r in sorted(rows, key=lambda r: (r["impl"], r["world"], r["tokens"])):
        got = r.get("nvlink_tx_bytes_per_op")
        if got is None or not r.get("correct"):
            continue
        exp = expected_tx_bytes(r["impl"] if r["impl"] != "ours:auto" else
                                "ours:" + next((k for k, v in VARIANTS.items()
                                                if v == (r.get("variant") or {}).get("variant")), "?"),
                                r["bytes"], r["world"])
        out.append(f"| {r['impl']} | {r['world']} | {r['tokens']} | {r['bytes'] >> 10} | {got / 1024:.1f} | "
                   + (f"{exp / 1024:.1f} | {got / exp:.2f} |" if exp else "- | - |"))
    return "\n".join(out)


def roofline_table(rows: list[dict], link_gbs: float | None = None) -> tuple[str, list[dict]]:
    """Achieved fraction of the NVLink roofline per size: the fused op has no FLOPs worth counting, so
    its target time is the bytes an all-reduce must move per GPU and direction without in-switch
    reduction, 2 (W - 1) / W S (a one-shot moves (W - 1) S; NVSwitch multicast needs only about S),
    at `link_gbs`. fraction = target / measured p50 of the fastest of our variants (and of the best
    baseline); small messages are latency-bound, which the fraction shows. `link_gbs` defaults to the
    measured per-direction peer copy of the newest committed platform record (utils.peaks.link_gbs)."""
    if link_gbs is None:
        from ..utils.peaks import link_gbs as measured_link_gbs

        link_gbs = measured_link_gbs()
    out = ["| world | tokens | KB | target us | best ours | us | fraction | best baseline | us | fraction |",
           "|---|---|---|---|---|---|---|---|---|---|"]
    summary = []
    for world in sorted({r["world"] for r in rows}):
        sub = [r for r in rows if r["world"] == world and r.get("correct") and r.get("p50_us")]
        for T in sorted({r["tokens"] for r in sub}):
            at = [r for r in sub if r["tokens"] == T]
            ours = min((r for r in at if r["impl"].startswith("ours") and r["impl"] != "ours:auto"),
                       key=lambda r: r["p50_us"], default=None)
            base = min((r for r in at if r["impl"] in BASELINES), key=lambda r: r["p50_us"], default=None)
            msg = at[0]["bytes"]
            target = 2 * (world - 1) / world * msg / (link_gbs * 1e3)  # us (GB/s = 1e3 bytes/us)
            fo = target / ours["p50_us"] if ours else None
            fb = target / base["p50_us"] if base else None
            out.append(f"| {world} | {T} | {msg >> 10} | {target:.2f} | " +
                       (f"{ours['impl']} | {ours['p50_us']:.2f} | {fo:.3f} | " if ours else "- | - | - | ") +
                       (f"{base['impl']} | {base['p50_us']:.2f} | {fb:.3f} |" if base else "- | - | - |"))
            summary.append(dict(world=world, tokens=T, bytes=msg, link_gbs=link_gbs, target_us=target,
                                ours=ours and ours["impl"], fraction=fo, baseline=base and base["impl"],
                                baseline_fraction=fb))
    return "\n".join(out), summary


def validate(rows: list[dict], tol: float = 0.03) -> list[dict]:
    """Check the variant table in fresh launches (the reference's validate step,
    exp/M18_incremental/run_b.py:60-76 and README.md:131-140): `rows` hold several independent sweeps,
    each with `ours:auto` (the table's choice) and the individual variants. Per (world, dtype, hidden,
    tokens): median [min, max] over launches of auto and of every fixed variant; `within` = auto is within
    `tol` of the best fixed variant's median; `retune` = a fixed variant beats auto by >= `tol` with
    disjoint [min, max] intervals over >= 3 launches (the only case in which the table entry changes)."""
    from ..utils.stats import disjoint, median_minmax

    out = []
    keys = sorted({(r["world"], r["dtype"], r["hidden"], r["tokens"]) for r in rows if r["impl"] == "ours:auto"})
    for w, dt, h, T in keys:
        at = [r for r in rows if (r["world"], r["dtype"], r["hidden"], r["tokens"]) == (w, dt, h, T)
              and r.get("correct") and r.get("p50_us")]
        per: dict[str, list[float]] = {}
        for r in at:
            if r["impl"].startswith("ours:"):
                per.setdefault(r["impl"], []).append(r["p50_us"])
        if "ours:auto" not in per:
            continue
        auto = median_minmax(per.pop("ours:auto"))
        if not per:
            continue
        stats = {k: median_minmax(v) for k, v in per.items()}
        best = min(stats, key=lambda k: stats[k]["med"])
        b = stats[best]
        gain = auto["med"] / b["med"] - 1.0
        out.append(dict(world=w, dtype=dt, hidden=h, tokens=T, auto=auto, best=best, best_stats=b, gain=gain,
                        within=gain <= tol,
                        retune=gain >= tol and disjoint(auto, b) and auto["n"] >= 3 and b["n"] >= 3))
    return out


def calibrate(rows: list[dict], table_path: Path | None = None) -> VariantTable:
    """Fastest correct variant (with its geometry) per (world, dtype, hidden, rows bucket)."""
    import torch

    t = VariantTable.load(table_path)
    for r in rows:
        if not r["impl"].startswith("ours:") or r["impl"] == "ours:auto" or not r["correct"] or not r["p50_us"]:
            continue
        dtype = getattr(torch, r["dtype"])
        key = VariantTable.key(r["world"], dtype, r["hidden"], r["tokens"])
        cur = t.entries.get(key)
        if cur is None or cur.p50_us is None or r["p50_us"] < cur.p50_us:
            v = r.get("variant") or {}
            t.entries[key] = Choice(VARIANTS[r["impl"].split(":", 1)[1]], v.get("blocks", 0), v.get("threads", 0),
                                    v.get("cluster", 0), round(r["p50_us"], 3))
    return t


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("sweeps", nargs="+")
    ap.add_argument("--calibrate", action="store_true", help="update the committed variant table")
    ap.add_argument("--table", default=None)
    ap.add_argument("--nvlink", action="store_true", help="measured vs expected NVLink bytes per call")
    ap.add_argument("--roofline", action="store_true", help="achieved fraction of the NVLink roofline per size")
    ap.add_argument("--validate", action="store_true",
                    help="the given sweeps are fresh launches with ours:auto: check the table (3 % rule)")
    ap.add_argument("--repeats", nargs=2, metavar=("OURS", "BASELINE"),
                    help="median [min, max] over the given sweeps (independent launches) and the effectiveness rule")
    a = ap.parse_args()
    rows = load(a.sweeps)
    if a.validate:
        print("| world | dtype | hidden | tokens | auto med [min, max] | best fixed | med [min, max] | auto slower by | "
              "within 3 % | retune |")
        print("|---|---|---|---|---|---|---|---|---|---|")
        for r in validate(rows):
            o, b = r["auto"], r["best_stats"]
            print(f"| {r['world']} | {r['dtype']} | {r['hidden']} | {r['tokens']} | {o['med']:.2f} [{o['lo']:.2f}, "
                  f"{o['hi']:.2f}] (n={o['n']}) | {r['best']} | {b['med']:.2f} [{b['lo']:.2f}, {b['hi']:.2f}] | "
                  f"{100 * r['gain']:+.1f}% | {'yes' if r['within'] else 'no'} | {'yes' if r['retune'] else 'no'} |")
        return
    if a.repeats:
        print(f"| world | tokens | {a.repeats[0]} med [min, max] | {a.repeats[1]} med [min, max] | gain | effective |")
        print("|---|---|---|---|---|---|")
        for r in repeats(rows, *a.repeats):
            o, b = r["ours"], r["base"]
            print(f"| {r['world']} | {r['tokens']} | {o['med']:.2f} [{o['lo']:.2f}, {o['hi']:.2f}] (n={o['n']}) | "
                  f"{b['med']:.2f} [{b['lo']:.2f}, {b['hi']:.2f}] (n={b['n']}) | {100 * r['gain']:+.1f}% | "
                  f"{'yes' if r['effective'] else 'no'} |")
        return
    if a.nvlink:
        print(link_table(rows))
        return
    if a.roofline:
        print(roofline_table(rows)[0])
        return
    text, _ = table(rows)
    print(text)
    if a.calibrate:
        from ..parallel.variant_table import DEFAULT_TABLE

        path = Path(a.table) if a.table else DEFAULT_TABLE
        t = calibrate(rows, path)
        t.save(path)
        print(f"\nvariant table: {len(t.entries)} entries -> {path}")


if __name__ == "__main__":
    main()
