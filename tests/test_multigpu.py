"""Multi-GPU tier: real one-process-per-GPU runs of the fused collective and the TP decode runner at 2, 4
and 8 ranks (each case skips when the node has fewer GPUs).

Each test launches `comm_opt_b200.harness.mp_selftest` under torch.distributed.run (127.0.0.1
rendezvous) with an outer `timeout -k 60`, and asserts on its JSON summary. What the parts check:

* functional: every variant (NVSwitch multicast forms included when the heap has a multicast object)
  x bf16 / fp16 / fp32 x several shapes against an fp32 NCCL oracle, the small all-gather, the
  interleaving test (60 calls of mixed token counts, block counts and variants, eager and CUDA-graph
  replay, the reference's exp/M16_epoch_fix/test_interleave.py sequence) and a rank launching late;
* decode / decode_fused / decode_fused_epi: the tiny Llama decode step (separate boundaries, fused
  layer boundaries, fused SiLU and RoPE epilogues) against the unsharded fp32 model;
* fault and leave: a rank skips a call (bounded waits time out, reset() recovers) and a rank leaves
  between steps (the others learn of it from the store before their next launch). Both run on the
  CUDA-IPC heap with NVLS off everywhere (NCCL_NVLS_ENABLE=0, no multicast object, plain peer loads);
  nothing faults or hangs a GPU.
"""
import json
import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT, free_port

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

WORLDS = [2, 4, 8]
NO_NVLS = {"NCCL_NVLS_ENABLE": "0"}


def _run(parts: str, nproc: int, extra_env: dict | None = None, limit: int = 600) -> dict:
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
    assert p.returncode == 0 and res["world"] == nproc
    return res


@pytest.mark.parametrize("world", WORLDS)
def test_fused_collective_functional(world):
    res = _run("functional", world)
    assert res["checks"] > 100


@pytest.mark.parametrize("world", WORLDS)
def test_tp_decode_matches_reference(world):
    _run("decode,decode_fused,decode_fused_epi", world)


@pytest.mark.parametrize("world", WORLDS)
def test_fault_injection_and_reset(world):
    _run("fault", world, extra_env=NO_NVLS, limit=300)


@pytest.mark.parametrize("world", WORLDS)
def test_rank_leaves_between_steps(world):
    _run("leave", world, extra_env=NO_NVLS, limit=300)
