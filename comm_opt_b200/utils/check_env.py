"""Machine check: what this framework needs (required) and what its baselines and GPU runs use
(optional), each probed and reported on one line, with the exit code telling whether the required
part is complete (the reference ships the same kind of check as env/check_env.py).

    python -m comm_opt_b200.utils.check_env          (no GPU work)
    python -m comm_opt_b200.utils.check_env --gpu    (also the 2-GPU self-test, bounded by a timeout)
"""
from __future__ import annotations

import importlib
import os
import shutil
import subprocess
import sys
from dataclasses import dataclass
from typing import Callable

from .results import ROOT


@dataclass
class Finding:
    item: str
    ok: bool
    detail: str
    required: bool
    remedy: str = ""

    @property
    def status(self) -> str:
        return "ok" if self.ok else ("FAIL" if self.required else "absent")


def _run(argv: list[str], limit: float = 120.0) -> tuple[int, str]:
    try:
        r = subprocess.run(argv, capture_output=True, text=True, timeout=limit)
        return r.returncode, (r.stdout + r.stderr).strip()
    except FileNotFoundError:
        return 127, "not found"
    except subprocess.TimeoutExpired:
        return 124, f"no answer within {limit:.0f} s"


def _module(name: str) -> tuple[bool, str]:
    try:
        m = importlib.import_module(name)
        return True, str(getattr(m, "__version__", getattr(m, "__file__", "?")))
    except Exception as e:  # noqa: BLE001 - any import failure means "absent"
        return False, f"{type(e).__name__}: {str(e)[:60]}"


def probe_toolchain() -> list[Finding]:
    import torch

    out = [Finding("torch", True, f"{torch.__version__} (CUDA {torch.version.cuda})", True)]
    rc, text = _run(["nvcc", "--version"])
    out.append(Finding("nvcc (sm_100a builds)", rc == 0, text.splitlines()[-1] if rc == 0 else text, True,
                       "a CUDA toolkit >= 12.8 on PATH"))
    ok, detail = _module("comm_opt_b200._C")
    out.append(Finding("native extension", ok, detail, True, "python setup.py build_ext --inplace"))
    for tool, req in (("git", True), ("ninja", True), ("ncu", False)):
        path = shutil.which(tool)
        out.append(Finding(tool, path is not None, path or "not on PATH", req, f"install {tool}"))
    return out


def probe_gpus() -> list[Finding]:
    import torch

    out = []
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    names = [torch.cuda.get_device_name(i) for i in range(n)]
    out.append(Finding("CUDA devices", n > 0, f"{n} x {names[0] if names else '-'}", False,
                       "kernels need an NVIDIA B200 (sm_100a)"))
    if n:
        caps = {torch.cuda.get_device_capability(i) for i in range(n)}
        out.append(Finding("compute capability 10.0", caps == {(10, 0)}, str(sorted(caps)), False,
                           "kernels are built for sm_100a only"))
        out.append(Finding("NCCL", True, ".".join(map(str, torch.cuda.nccl.version())), False))
        if n > 1:
            rc, topo = _run(["nvidia-smi", "topo", "-m"])
            links = topo.count("NV18") if rc == 0 else 0
            out.append(Finding("NVLink 5 between every pair", links >= n * (n - 1), f"{links} NV18 entries", False,
                               "expected NV18 between every pair of GPUs (NVSwitch)"))
    return out


def probe_baselines() -> list[Finding]:
    out = []
    for mod, role in (("vllm", "baselines vllm_car / nccl_norm"), ("flashinfer", "baselines trt_oneshot / trt_twoshot"),
                      ("pynvml", "NVLink counters, GPU state per launch")):
        ok, detail = _module(mod)
        out.append(Finding(mod, ok, detail if ok else f"{detail} ({role})", False))
    ref = ROOT / "baseline" / "_ref" / "exp"
    out.append(Finding("reference prototype source", ref.exists(), str(ref), False,
                       "a copy of the reference tree for the ref_m16nf baseline"))
    return out


def probe_selftest() -> list[Finding]:
    import torch

    if torch.cuda.device_count() < 2:
        return [Finding("2-GPU self-test", False, "skipped: fewer than 2 GPUs", False)]
    argv = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
            "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29699", "-m",
            "comm_opt_b200.harness.mp_selftest", "--parts", "functional"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    try:
        r = subprocess.run(argv, capture_output=True, text=True, cwd=ROOT, env=env, timeout=700)
        rc, text = r.returncode, r.stdout + r.stderr
    except subprocess.TimeoutExpired:
        rc, text = 124, ""
    verdicts = [l for l in text.splitlines() if l.startswith("{")]
    ok = rc == 0 and bool(verdicts) and '"ok": true' in verdicts[-1]
    return [Finding("2-GPU self-test", ok, (verdicts[-1] if verdicts else text[-160:])[:120], True,
                    "read the self-test output")]


def render(findings: list[Finding]) -> str:
    width = max(len(f.item) for f in findings)
    lines = []
    for f in findings:
        lines.append(f"[{f.status:>6}] {f.item:<{width}}  {f.detail}")
        if not f.ok and f.remedy:
            lines.append(f"         {'':<{width}}  needs: {f.remedy}")
    missing = [f.item for f in findings if f.required and not f.ok]
    optional = sum(1 for f in findings if not f.required and not f.ok)
    lines.append("")
    lines.append(f"required: {'complete' if not missing else 'incomplete - ' + '; '.join(missing)}"
                 f" | optional items absent: {optional}")
    return "\n".join(lines)


def main(argv: list[str]) -> int:
    groups: list[Callable[[], list[Finding]]] = [probe_toolchain, probe_gpus, probe_baselines]
    if "--gpu" in argv:
        groups.append(probe_selftest)
    findings = [f for g in groups for f in g()]
    print(render(findings))
    return 0 if all(f.ok for f in findings if f.required) else 1


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
