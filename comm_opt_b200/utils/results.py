"""Results directory contract: ``results/<exp>/<timestamp>/`` holding ``env.txt`` (environment
snapshot), ``schedule.tsv`` (executed order with GPU state before each job, start time, duration,
return code) and one JSON per job - the same contract as the reference's experiment runner
(exp/lib/ncclrun.py:55-106, results/<exp>/<ts>/ with env.txt and schedule.tsv).
"""
from __future__ import annotations

import json
import os
import shlex
import subprocess
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]


def _sh(cmd: str) -> str:
    try:
        return subprocess.run(cmd, shell=True, capture_output=True, text=True, timeout=30).stdout
    except (OSError, subprocess.TimeoutExpired):
        return ""


def env_snapshot() -> str:
    """Date, host, GPUs (driver, clocks, temperatures), NVLink topology, CUDA / NCCL / torch versions,
    git commit of this repository."""
    import torch

    parts = [
        "date: " + time.strftime("%Y-%m-%dT%H:%M:%S%z"),
        "host: " + os.uname().nodename,
        _sh("nvidia-smi --query-gpu=index,name,driver_version,clocks.sm,clocks.max.sm,clocks.mem,temperature.gpu,"
            "power.draw,power.limit --format=csv"),
        _sh("nvidia-smi topo -m"),
        "nvcc: " + _sh("nvcc --version | tail -1"),
        f"torch: {torch.__version__} cuda {torch.version.cuda} nccl "
        f"{'.'.join(map(str, torch.cuda.nccl.version())) if torch.cuda.is_available() else 'n/a'}",
        "git: " + _sh(f"git -C {shlex.quote(str(ROOT))} log -1 --format='%H %s'"),
        "env: " + " ".join(f"{k}={v}" for k, v in sorted(os.environ.items())
                           if k.startswith(("NCCL_", "CUDA_", "COB_", "TORCH_NCCL"))),
    ]
    return "\n".join(p.rstrip() for p in parts) + "\n"


def gpu_state() -> str:
    """SM clock (MHz), temperature (C) and power (W) of every GPU, read through NVML, as
    'clock/temp/power' per GPU joined by ';' ('' when NVML cannot be read)."""
    try:
        import pynvml

        pynvml.nvmlInit()
    except Exception:
        return ""
    parts = []
    try:
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            clk = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
            temp = pynvml.nvmlDeviceGetTemperature(h, pynvml.NVML_TEMPERATURE_GPU)
            watts = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
            parts.append(f"{clk}/{temp}/{watts:.0f}")
    except Exception:
        pass
    finally:
        pynvml.nvmlShutdown()
    return ";".join(parts)


class RunDir:
    def __init__(self, exp: str, base: Path | None = None, ts: str | None = None):
        self.path = (base or ROOT / "results") / exp / (ts or time.strftime("%Y%m%d_%H%M%S"))
        self.path.mkdir(parents=True, exist_ok=True)
        self._sched = None

    @classmethod
    def at(cls, path: Path) -> "RunDir":
        """An existing run directory (to resume a plan into it)."""
        path = Path(path)
        if not path.is_dir():
            raise FileNotFoundError(path)
        obj = cls.__new__(cls)
        obj.path, obj._sched = path, None
        return obj

    def snapshot(self):
        (self.path / "env.txt").write_text(env_snapshot())

    def schedule(self, order: int, tag: str, started: float, seconds: float, rc: int, state: str = "", **kw):
        new = not (self.path / "schedule.tsv").exists()
        with open(self.path / "schedule.tsv", "a") as f:
            if new:
                f.write("order\ttag\tgpu_state_before\tstart\tseconds\trc\textra\n")
            f.write(f"{order}\t{tag}\t{state}\t{time.strftime('%H:%M:%S', time.localtime(started))}\t{seconds:.1f}\t"
                    f"{rc}\t{json.dumps(kw) if kw else ''}\n")

    def write_json(self, name: str, obj):
        (self.path / name).write_text(json.dumps(obj, indent=1))

    def done(self, name: str) -> bool:
        """Cheap resume: a job whose result file exists in this run directory is skipped."""
        return (self.path / name).exists()
