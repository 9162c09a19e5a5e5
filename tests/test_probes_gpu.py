"""Primitive probes on one GPU (ranks emulated in one launch)."""
import pytest
import torch

from comm_opt_b200.harness.probes import VARIANTS, clock_mhz, run_rs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("variant", list(VARIANTS))
def test_rs_atomic_emulated(cuda, world, variant):
    r = run_rs(world, 8192, variant, cuda, emulate=True, blocks=16, reps=2)
    assert not r["timeout"]
    assert r["rel_err"] <= (1e-5 if variant <= 1 else 2 ** -5), r


def test_clock_calibration(cuda):
    mhz = clock_mhz(0, ns=5_000_000)
    assert 100 < mhz < 3000
