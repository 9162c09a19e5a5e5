"""Typed configuration of a TPCommunicator (one dataclass, overridable from the environment or a dict)."""
from __future__ import annotations

import os
from dataclasses import asdict, dataclass, fields


@dataclass
class CommConfig:
    max_rows: int = 512          # largest token count per call (decode batch)
    max_hidden: int = 8192       # largest row width (elements)
    max_gather: int = 4096       # largest small all-gather (32-bit words)
    timeout_ms: float = 1000.0   # bound of every device-side wait
    pdl: bool = True             # programmatic dependent launch
    allow_nvls: bool = True      # use NVSwitch multicast variants when the heap has a multicast object
    backend: str = "symm_mem"    # symmetric heap: "symm_mem" (multicast-capable) or "ipc"

    ENV = {"max_rows": "COB_MAX_ROWS", "max_hidden": "COB_MAX_HIDDEN", "max_gather": "COB_MAX_GATHER",
           "timeout_ms": "COB_WAIT_TIMEOUT_MS", "pdl": "COB_PDL", "allow_nvls": "COB_ALLOW_NVLS",
           "backend": "COB_HEAP_BACKEND"}

    def __post_init__(self):
        if self.max_rows <= 0 or self.max_hidden <= 0 or self.max_gather <= 0 or self.timeout_ms <= 0:
            raise ValueError(f"capacities and timeout must be positive: {self}")
        if self.backend not in ("symm_mem", "ipc"):
            raise ValueError(f"backend must be symm_mem or ipc, got {self.backend!r}")

    @classmethod
    def from_dict(cls, d: dict) -> "CommConfig":
        names = {f.name for f in fields(cls)}
        unknown = set(d) - names
        if unknown:
            raise ValueError(f"unknown communicator settings: {sorted(unknown)}")
        return cls(**d)

    @classmethod
    def from_env(cls, base: "CommConfig | None" = None, env=None) -> "CommConfig":
        """`base` (or the defaults) with every COB_* variable that is set applied on top."""
        env = os.environ if env is None else env
        d = asdict(base or cls())
        for f in fields(cls):
            key = cls.ENV.get(f.name)
            if key and key in env:
                raw = env[key]
                if f.type in ("bool", bool):
                    d[f.name] = raw.strip().lower() in ("1", "true", "yes", "on")
                elif f.type in ("int", int):
                    d[f.name] = int(raw)
                elif f.type in ("float", float):
                    d[f.name] = float(raw)
                else:
                    d[f.name] = raw
        return cls(**d)

    def kwargs(self) -> dict:
        """Keyword arguments of TPCommunicator."""
        return asdict(self)
