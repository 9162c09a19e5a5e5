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


@pytest.mark.skipif(not available(), reason="native extension not built")
@pytest.mark.parametrize("model", ["70b", "8b"])
@pytest.mark.parametrize("tp", [2, 4, 8])
def test_fused_gemm_plans_for_decode_shapes(model, tp):
    """Every layer-boundary GEMM of a TP decode step gets a launchable plan: consumer grids resident at
    once (<= SMs x CTAs per SM) and within the per-block epoch words, split-K only with one tile per
    CTA, the per-piece sum-of-squares buffer within shared memory, paired epilogues 2..8 splits or none."""
    from comm_opt_b200._ext import native
    from comm_opt_b200.models.llama import PRESETS

    C = native()
    cfg = PRESETS[model]
    s = cfg.shard(tp)
    D, H = cfg.head_dim, cfg.hidden
    sms = 148
    for B in (1, 8, 32, 64, 128):
        for N, K in ((H, s["nq"] * D), (H, s["inter"])):  # o_proj, down_proj: push GEMMs
            bn, tiles, splits, kps, xctas, ctas, smem = C.fused_gemm_plan(B, N, K, 0, sms, False, 0)
            assert splits >= 1 and xctas == tiles and ctas == tiles * splits and 128 % (8 * splits) == 0
            assert kps * (splits - 1) < K // 64 and smem <= 227 * 1024
        for N, epi in ((2 * s["inter"], 1), ((s["nq"] + 2 * s["nkv"]) * D, 2), (s["vocab"], 0)):
            for e in {0, epi}:
                bn, tiles, splits, kps, xctas, ctas, smem = C.fused_gemm_plan(B, N, H, 0, sms, True, e)
                cap = min(sms * (2 if bn <= 64 else 1), C.kMaxBlocks)
                if e and splits == 0:
                    continue  # the paired epilogue is not offered for this shape: separate kernels run
                assert 1 <= splits <= (8 if e else 16) and ctas == xctas * splits <= cap
                assert ctas <= C.kMaxPieces and (splits == 1 or xctas == tiles)
                if e:
                    assert splits >= 2 and xctas == tiles
                KV = H // 8
                slen = min(KV, kps * 8)
                assert B * (-(-slen // xctas) + 1) <= 2048, (B, N, splits, xctas)


def test_error_word_decoding():
    from comm_opt_b200.parallel.communicator import decode_state, describe_error

    # lamport_1s (variant 1) phase 2 timed out on row 3, vector 17, waiting for peer 5 in call 42
    words = [41, (1 << 32) | 0, (1 << 32) | 2, (3 << 32) | 17, 5, 42]
    st = decode_state(words, 0)
    assert st["error"] == 1 and st["reasons"] == ["timeout waiting for landing data"]
    assert st["where"]["kernel"] == "lamport_1s" and st["where"]["row"] == 3 and st["where"]["vector"] == 17
    msg = describe_error(st)
    assert "lamport_1s phase 2" in msg and "peer/block 5" in msg and "call 42" in msg
    # fused GEMM family, error bits combined, a negative int64 word (bit 63 set) decodes unsigned
    st = decode_state([7, (9 << 32) | 0, 0xF6 << 32, -1, 3, 8], 2)
    assert st["where"]["kernel"] == "fused_gemm" and st["error"] == 9 and len(st["reasons"]) == 2
    assert st["where"]["row"] == 0xFFFFFFFF
    assert decode_state([0, 0, 0, 0, 0, 0], 1)["reasons"] == []


@pytest.mark.skipif(not available(), reason="native extension not built")
def test_fused_ar_geometry_rules():
    """resolve_config (host C++) over worlds, dtypes, sizes and variants: every accepted geometry is
    launchable (blocks within the per-rank SM budget and the barrier slots, cluster divides the grid,
    a row chunk fits the threads); rejections only where a variant cannot run."""
    from comm_opt_b200._ext import native

    C = native()
    esz = {0: 4, 1: 2, 2: 2}
    for world in (2, 4, 8):
        for dtype in (0, 1, 2):
            L = C.plan_layout(world, 512, 8192 if dtype else 4096, esz[dtype], 4096)
            for emulate in (0, 1):
                budget = 148 // (world if emulate else 1)
                for hidden in (1024, 2048, 4096, 5120, 6400, 6656, 8192):
                    hv = hidden * esz[dtype] // 16
                    if hv > L[14]:
                        continue
                    for rows in (1, 3, 8, 17, 64, 512):
                        for v in range(1, 8):
                            for mc in (False, True):
                                rc, var, b, t, cl = C.fused_ar_config(L, world, rows, hidden, dtype, v, 0, 0, 0,
                                                                      emulate, 148, mc)
                                nvls = v in (3, 4)
                                two = v in (2, 4, 6)
                                if nvls and not mc:
                                    assert rc != 0
                                    continue
                                if two and (hv % world or hv % 32):
                                    assert rc != 0
                                    continue
                                assert rc == 0, (world, dtype, emulate, hidden, rows, v)
                                assert 1 <= b <= min(budget, C.kMaxBlocks) and t % 32 == 0 and t <= 512
                                if two:
                                    assert cl == 1 and t <= 256
                                else:
                                    assert cl in (1, 2, 4, 8) and b % cl == 0
                                    assert -(-hv // cl) <= t * 4


@pytest.mark.skipif(not available(), reason="native extension not built")
def test_committed_variant_table_geometries_resolve():
    """Every entry of the committed, measured variant table is accepted by the current kernels."""
    from comm_opt_b200._ext import native
    from comm_opt_b200.parallel.variant_table import VariantTable

    C = native()
    t = VariantTable.load()
    for key, ch in t.entries.items():
        w, dt, h, tb = key.split("/")
        world, hidden = int(w[1:]), int(h[1:])
        dtype = {"float32": 0, "float16": 1, "bfloat16": 2}[dt]
        rows = int(tb[1:])
        esize = 4 if dtype == 0 else 2
        L = C.plan_layout(world, 512, hidden, esize, 4096)
        rc, *_ = C.fused_ar_config(L, world, rows, hidden, dtype, ch.variant, ch.blocks, ch.threads, ch.cluster,
                                   0, 148, True)
        assert rc == 0, (key, ch)


@pytest.mark.skipif(not available(), reason="native extension not built")
def test_streamk_gemm_plans():
    """Stream-K partition of every decode projection (70B / 8B, TP 1/2/4/8, batch 1..256): CTAs within
    the SMs and the flattened work, at most 48 contributors per split tile, batch tile covering M."""
    from comm_opt_b200._ext import native
    from comm_opt_b200.models.llama import PRESETS

    C = native()
    for model in ("70b", "8b"):
        cfg = PRESETS[model]
        for tp in (1, 2, 4, 8):
            s = cfg.shard(tp)
            D, H = cfg.head_dim, cfg.hidden
            shapes = [((s["nq"] + 2 * s["nkv"]) * D, H), (H, s["nq"] * D), (2 * s["inter"], H), (H, s["inter"]),
                      (s["vocab"], H)]
            for M in (1, 8, 32, 64, 128, 256):
                for N, K in shapes:
                    bn, tiles, ctas, ws = C.gemm_plan(M, N, K, 148, 0)
                    KT = -(-K // 64)
                    total = tiles * KT
                    assert bn >= M and bn in (16, 32, 64, 128, 256)
                    assert tiles == -(-N // 128) and 1 <= ctas <= min(148, total)
                    assert -(-KT * ctas // total) + 1 <= 48
                    assert ws == ctas * 2 * 128 * bn * 4


@pytest.mark.skipif(not available(), reason="native extension not built")
def test_primitive_probe_heap_and_multicast_modes():
    """Probe heap regions in order (epochs, flags, multicast-barrier counters, stage, landing) and large
    enough; the NVSwitch modes are refused without real ranks (no multicast object when emulated)."""
    from comm_opt_b200._ext import native
    from comm_opt_b200.harness.probes import NVLS_MODES, PRIM_MODES, run_prim

    for world in (2, 4, 8):
        n = 4096 * world
        total, f, st, land, nv = native().prim_layout(world, n)
        assert 0 < f < nv < st < land < total
        assert nv - f >= 8 * 256 * 8 and st - nv >= 8 * 256 and land - st >= 2 * n * 4
        assert total - land >= 2 * 8 * (n // world) * 4
    assert {PRIM_MODES[m] for m in NVLS_MODES} == {"rs_nvls", "ag_nvls"}
    r = run_prim(4, 4096 * 4, 4, "cpu", emulate=True)
    assert r["skip"] and r["mode"] == "rs_nvls"
