"""Multi-GPU tier: real one-process-per-GPU runs of the fused collective and the TP decode runner.

Each test launches `comm_opt_b200.harness.mp_selftest` under torch.distributed.run on 2 GPUs
(127.0.0.1 rendezvous) with an outer `timeout -k 60`, and asserts on its JSON summary. The
fault-injection run keeps NVLS off everywhere (NCCL_NVLS_ENABLE=0, CUDA-IPC heap without a
multicast object, plain peer loads).
"""
import json
import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT, free_port

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _run(parts: str, nproc: int = 2, extra_env: dict | None = None, limit: int = 600) -> dict:
    if torch.cuda.device_count() < nproc:
        pytest.skip(f"needs {nproc} GPUs")
    env = dict(os.environ, **(extra_env or {}))
    cmd = ["timeout", "-k", "60", str(limit), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={free_port()}",
           "-m", "comm_opt_b200.harness.mp_selftest", "--parts", parts]
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert lines, f"no summary (rc={p.returncode}):\n{p.stdout[-3000:]}\n{p.stderr[-3000:]}"
    res = json.loads(lines[-1])
    assert res["ok"], res["failures"]
    assert p.returncode == 0
    return res


def test_fused_collective_two_ranks():
    res = _run("functional")
    assert res["checks"] > 100


def test_tp2_decode_matches_reference():
    _run("decode")


def test_fault_injection_and_reset():
    _run("fault", extra_env={"NCCL_NVLS_ENABLE": "0"}, limit=300)
