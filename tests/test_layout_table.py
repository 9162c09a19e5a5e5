"""Heap layout planning and the variant table (no GPU)."""
import json

import pytest
import torch

from comm_opt_b200._ext import available
from comm_opt_b200.parallel.symm import plan_layout_py
from comm_opt_b200.parallel.variant_table import VARIANTS, Choice, VariantTable, rows_bucket


@pytest.mark.parametrize("world,rows,hidden,esize", [(2, 64, 4096, 4), (8, 512, 8192, 2), (4, 128, 5120, 2)])
def test_layout_regions_disjoint(world, rows, hidden, esize):
    L = plan_layout_py(world, rows, hidden, esize, 4096)
    order = ["state", "flags", "nvls", "land1", "rs", "ag", "agp", "stage", "hbuf", "hpart", "gather"]
    offs = [getattr(L, k) for k in order] + [L.total]
    assert offs == sorted(offs) and len(set(offs)) == len(offs)
    assert all(o % 4096 == 0 for o in offs[:-1]) and L.total % (2 << 20) == 0
    hv = hidden * esize // 16
    assert L.rs - L.land1 >= 2 * world * rows * hv * 16
    assert L.max_hv == hv and L.sv_max * world >= hv


@pytest.mark.skipif(not available(), reason="native extension not built")
def test_layout_python_matches_native():
    from comm_opt_b200._ext import native

    for args in [(2, 64, 4096, 4, 128), (8, 512, 8192, 2, 4096), (4, 7, 5120, 2, 64)]:
        assert list(native().plan_layout(*args)) == plan_layout_py(*args).as_list()


def test_variant_rule_and_roundtrip(tmp_path):
    t = VariantTable()
    assert t.lookup(8, torch.bfloat16, 2, 8192, 1, False).variant == VARIANTS["lamport_1s"]
    assert t.lookup(8, torch.bfloat16, 2, 8192, 512, False).variant == VARIANTS["lamport_2s"]
    t.set(8, torch.bfloat16, 8192, 16, Choice(VARIANTS["nvls_1s"], 16, 256, 2, 3.5))
    # an NVLS entry is ignored where multicast is unavailable
    assert t.lookup(8, torch.bfloat16, 2, 8192, 9, False).variant != VARIANTS["nvls_1s"]
    assert t.lookup(8, torch.bfloat16, 2, 8192, 9, True).variant == VARIANTS["nvls_1s"]
    p = tmp_path / "t.json"
    t.save(p)
    t2 = VariantTable.load(p)
    assert t2.entries == t.entries and json.loads(p.read_text())
    assert [rows_bucket(r) for r in (1, 2, 3, 5, 64, 65)] == [1, 2, 4, 8, 64, 128]
