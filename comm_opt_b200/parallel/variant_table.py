"""Per-size choice of the fused all-reduce variant and launch geometry.

The reference fixed one structure (pull reduce-scatter + LL128 push all-gather) and a block count
per size measured by a calibrate run and checked by a separate validation run
(exp/M18_incremental/run_b.py:60-76, table JSON `--table` in exp/M18_incremental/bench_inc.py).
Here the table key is (world, dtype, hidden, rows bucket) and the value names the variant
(one-shot push / two-shot push / NVLS / pull) and its geometry, produced by
``comm_opt_b200.harness.sweep --calibrate`` from measured p50 device latency. Until a table has
been measured for a configuration, a size rule picks the variant.
"""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass
from pathlib import Path

VARIANTS = {"lamport_1s": 1, "lamport_2s": 2, "nvls_1s": 3, "nvls_2s": 4, "pull_1s": 5, "pull_2s": 6,
            "lamport_1sx": 7}
VARIANT_NAMES = {v: k for k, v in VARIANTS.items()}
NVLS_VARIANTS = {3, 4}
TWO_SHOT = {2, 4, 6}

DEFAULT_TABLE = Path(__file__).with_name("variant_table.json")


@dataclass
class Choice:
    variant: int
    blocks: int = 0     # 0 = kernel's own rule
    threads: int = 0
    cluster: int = 0
    p50_us: float | None = None  # measured latency that selected it (None = rule)


def rows_bucket(rows: int) -> int:
    """Power-of-two bucket (1, 2, 4, ...) containing `rows`."""
    b = 1
    while b < rows:
        b *= 2
    return b


def dtype_name(dtype) -> str:
    s = str(dtype)
    return s.split(".")[-1]


class VariantTable:
    def __init__(self, entries: dict | None = None):
        self.entries: dict[str, Choice] = {}
        for k, v in (entries or {}).items():
            self.entries[k] = v if isinstance(v, Choice) else Choice(**v)

    @staticmethod
    def key(world: int, dtype, hidden: int, rows: int) -> str:
        return f"w{world}/{dtype_name(dtype)}/h{hidden}/t{rows_bucket(rows)}"

    @staticmethod
    def rule(world: int, esize: int, hidden: int, rows: int, have_nvls: bool) -> Choice:
        """Size rule used before calibration: one-shot push for small messages, two-shot push above.

        One-shot moves (world-1)*M bytes per rank in one hop; two-shot moves 2*(world-1)/world*M in
        two hops, so it wins once the message is bandwidth-bound.
        """
        nbytes = rows * hidden * esize
        hv = hidden * esize // 16
        two_ok = hv % world == 0 and hv % 32 == 0
        if nbytes <= (256 << 10) or not two_ok:
            return Choice(VARIANTS["lamport_1s"])
        return Choice(VARIANTS["lamport_2s"])

    def lookup(self, world: int, dtype, esize: int, hidden: int, rows: int, have_nvls: bool) -> Choice:
        c = self.entries.get(self.key(world, dtype, hidden, rows))
        if c is not None and (c.variant not in NVLS_VARIANTS or have_nvls):
            return c
        return self.rule(world, esize, hidden, rows, have_nvls)

    def set(self, world: int, dtype, hidden: int, rows: int, choice: Choice):
        self.entries[self.key(world, dtype, hidden, rows)] = choice

    def save(self, path: str | Path):
        Path(path).write_text(json.dumps({k: asdict(v) for k, v in sorted(self.entries.items())}, indent=1))

    @classmethod
    def load(cls, path: str | Path | None = None) -> "VariantTable":
        p = Path(path) if path else DEFAULT_TABLE
        if not p.exists():
            return cls()
        return cls(json.loads(p.read_text()))
