"""Check this machine against what the framework needs and say what is missing (the reference's
env/check_env.py:18-123: table of OK / MISSING / optional rows, exit code, optional GPU smoke test).

    python -m comm_opt_b200.utils.check_env          (no GPU work)
    python -m comm_opt_b200.utils.check_env --gpu    (also runs the 2-GPU self-test, bounded by a timeout)
"""
from __future__ import annotations

import importlib
import shutil
import subprocess
import sys

from .results import ROOT

rows: list[tuple] = []
failed: list[str] = []


def sh(cmd: str) -> tuple[int, str]:
    try:
        r = subprocess.run(cmd, shell=True, capture_output=True, text=True, timeout=120)
        return r.returncode, (r.stdout + r.stderr).strip()
    except subprocess.TimeoutExpired:
        return 124, "timeout"


def check(name: str, ok: bool, found: str, hint: str = "", required: bool = True):
    rows.append(("OK" if ok else ("MISSING" if required else "optional"), name, found, "" if ok else hint))
    if required and not ok:
        failed.append(name)


def main(argv: list[str]) -> int:
    import torch

    check("torch", True, f"{torch.__version__} (cuda {torch.version.cuda})")
    rc, out = sh("nvcc --version")
    check("nvcc (sm_100a builds)", rc == 0, out.splitlines()[-1] if rc == 0 else "not found", "install CUDA >= 12.8")
    try:
        C = importlib.import_module("comm_opt_b200._C")
        check("native extension", True, C.__file__)
    except Exception as e:
        check("native extension", False, str(e)[:80], "python setup.py build_ext --inplace")
    rc, out = sh("nvidia-smi --query-gpu=name,driver_version --format=csv,noheader")
    gpus = [l for l in out.splitlines() if l.strip()] if rc == 0 else []
    check("GPUs", bool(gpus), f"{len(gpus)}x {gpus[0] if gpus else '-'}", "needs NVIDIA B200 (sm_100a)",
          required=False)
    if gpus:
        check("B200", all("B200" in g for g in gpus), gpus[0], "kernels are built for sm_100a only", required=False)
        rc, topo = sh("nvidia-smi topo -m")
        nv = topo.count("NV18")
        check("NVLink 5 topology", nv >= len(gpus) * (len(gpus) - 1) or len(gpus) == 1,
              f"{nv} NV18 entries", "expected NV18 between every pair of GPUs", required=False)
    if torch.cuda.is_available():
        check("NCCL", True, ".".join(map(str, torch.cuda.nccl.version())))
    for mod, why in (("vllm", "baseline vllm_car / nccl_norm (fused_add_rms_norm)"),
                     ("flashinfer", "baseline trt_oneshot / trt_twoshot")):
        try:
            m = importlib.import_module(mod)
            check(mod, True, getattr(m, "__version__", "?"), why, required=False)
        except Exception as e:
            check(mod, False, type(e).__name__, why, required=False)
    check("reference prototype source", (ROOT / "baseline" / "_ref" / "exp").exists(), "baseline/_ref/exp",
          "copy of the reference tree for the ref_m16nf baseline", required=False)
    for tool in ("ncu", "git", "ninja"):
        check(tool, shutil.which(tool) is not None, shutil.which(tool) or "not found", f"install {tool}",
              required=tool != "ncu")
    if "--gpu" in argv:
        if torch.cuda.device_count() < 2:
            check("GPU smoke test (2-GPU self-test)", False, "skipped: fewer than 2 GPUs", "", required=False)
        else:
            rc, out = sh(f"cd {ROOT} && NCCL_NVLS_ENABLE=0 timeout -k 60 600 {sys.executable} -m torch.distributed.run "
                         "--nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 --master-port 29699 "
                         "-m comm_opt_b200.harness.mp_selftest --parts functional")
            last = [l for l in out.splitlines() if l.startswith("{")]
            check("GPU smoke test (2-GPU self-test)", rc == 0 and bool(last) and '"ok": true' in last[-1],
                  last[-1][:120] if last else out[-200:], "see the self-test output")
    w = max(len(r[1]) for r in rows)
    for status, name, found, hint in rows:
        print(f"{status:8s} {name:<{w}}  {found}" + (f"\n{'':8s} {'':<{w}}  -> {hint}" if hint else ""))
    print(f"\n{'ALL REQUIRED ITEMS OK' if not failed else 'MISSING REQUIRED: ' + ', '.join(failed)}")
    return 1 if failed else 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
