"""Measured denominators of the roofline fractions.

* HBM: `hbm_gbs()` reads MEASURED_PEAKS.json (a STREAM-style copy measured on this pool's B200s).
* NVLink: `link_gbs()` reads the newest committed results/platform/<ts>/link.json written by
  `python -m comm_opt_b200.harness.platform_peaks` (GPU 0 -> peer copy of 1 GiB, median over peers,
  bytes per direction). There is no constant fallback: without a record the caller is told to run
  the measurement.
"""
from __future__ import annotations

import json
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]


class NoRecord(RuntimeError):
    pass


def hbm_gbs(path: Path | None = None) -> float:
    p = Path(path or ROOT / "MEASURED_PEAKS.json")
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, KeyError, ValueError) as e:
        raise NoRecord(f"no HBM copy bandwidth in {p}: {e}") from e


def latest_link_record(base: Path | None = None) -> Path:
    runs = sorted(Path(base or ROOT / "results" / "platform").glob("*/link.json"))
    if not runs:
        raise NoRecord("no results/platform/*/link.json: run python -m comm_opt_b200.harness.platform_peaks")
    return runs[-1]


def link_gbs(base: Path | None = None) -> float:
    """Measured NVLink bytes per direction per GPU (GB/s): median GPU 0 -> peer copy of the newest record."""
    path = latest_link_record(base)
    rec = json.loads(path.read_text())
    if "peer_copy_gbs_median" not in rec:
        raise NoRecord(f"{path} has no peer copy (measured on one GPU)")
    return float(rec["peer_copy_gbs_median"])
