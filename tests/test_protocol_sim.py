"""Host-side model checking of the synchronisation protocol (no GPU)."""
import pytest

from comm_opt_b200.parallel.protocol_sim import (L1S, L1SX, L2S, P1S, P2S, Call, ProtocolViolation, random_calls,
                                                 simulate, simulate_cluster_exchange)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_random_interleavings(world):
    for seed in range(4):
        res = simulate(world, random_calls(24, seed + 10 * world), seed=seed)
        assert res["epochs"] == [24] * world


@pytest.mark.parametrize("variant", [L1S, L2S, P1S, P2S, L1SX])
def test_slow_rank_each_variant(variant):
    calls = [Call(variant, b, t) for b, t in [(1, 1), (4, 8), (2, 3), (8, 8), (1, 5)] * 3]
    for slow in range(4):
        simulate(4, calls, seed=slow, slow_rank=slow, slow_factor=50)


def test_mixed_grids_like_graph_per_batch():
    # one CUDA graph per batch size, replayed in random order: grid sizes differ call to call
    calls = random_calls(40, 3, rows=(1, 2, 8, 13), blocks=(1, 3, 8))
    simulate(8, calls, seed=5, slow_rank=7)


def test_checker_detects_single_slot_protocol():
    caught = 0
    for seed in range(6):
        try:
            simulate(4, random_calls(20, seed), seed=seed, slow_rank=1, nslots=1)
        except ProtocolViolation:
            caught += 1
    assert caught == 6


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_boundary_mixed_with_fused_ar(world):
    """gemm_push + ar_norm_gemm calls share the epoch and land1 with the standalone one-shot calls."""
    from comm_opt_b200.parallel.protocol_sim import FG

    for seed in range(3):
        calls = random_calls(16, seed + 100 * world, variants=(L1S, FG, L2S, FG))
        res = simulate(world, calls, seed=seed, slow_rank=seed % world)
        assert res["epochs"] == [16] * world


def test_checker_detects_single_slot_fused_boundary():
    from comm_opt_b200.parallel.protocol_sim import FG

    caught = 0
    for seed in range(6):
        try:
            simulate(4, [Call(FG, 2, 2, 2)] * 12, seed=seed, slow_rank=seed % 4, slow_factor=40, nslots=1)
        except ProtocolViolation:
            caught += 1
    assert caught >= 5


@pytest.mark.parametrize("world", [2, 4, 8])
def test_nvls_variants_mixed(world):
    """Multicast-barrier variants (in-switch reduce, multicast store of h) mixed with every other
    variant, different grid sizes per call, a slow rank."""
    from comm_opt_b200.parallel.protocol_sim import NV1S, NV2S

    for seed in range(2):
        calls = random_calls(12, seed + 7 * world, variants=(NV1S, NV2S, L1S, P2S, NV2S), rows=(1, 3, 8),
                             blocks=(1, 2, 3))
        res = simulate(world, calls, seed=seed, slow_rank=(seed + 1) % world, slow_factor=30)
        assert res["epochs"] == [12] * world


def test_checker_detects_single_stage_slot_nvls():
    from comm_opt_b200.parallel.protocol_sim import NV1S, NV2S

    caught = 0
    for seed in range(4):
        try:
            simulate(4, [Call(NV1S, 2, 3), Call(NV2S, 1, 3)] * 6, seed=seed, slow_rank=seed, slow_factor=40, nslots=1)
        except ProtocolViolation:
            caught += 1
    assert caught >= 3


def test_deferred_restore_mixed_with_one_shot():
    """Landing cells given back after the row is finished (lamport_1sx) interleaved with the
    restore-at-read one-shot and the two-shot calls on the same landing buffers, a slow rank."""
    for world in (2, 4, 8):
        for seed in range(3):
            calls = random_calls(18, seed + 31 * world, variants=(L1SX, L1S, L1SX, L2S))
            res = simulate(world, calls, seed=seed, slow_rank=(seed + 1) % world, slow_factor=40)
            assert res["epochs"] == [18] * world


@pytest.mark.parametrize("ctas", [2, 4, 8, 16])
def test_cluster_exchange(ctas):
    """Row sums exchanged through per-CTA shared-memory words with two slots (row_sum_xch)."""
    for rows in (1, 3, 9):
        for seed in range(4):
            res = simulate_cluster_exchange(ctas, rows, seed=seed, slow=seed % ctas, slow_factor=30)
            assert res["sums"] == [sum(c * 1000 + it for c in range(ctas)) for it in range(rows)]


def test_checker_detects_single_slot_cluster_exchange():
    caught = 0
    for seed in range(6):
        try:
            simulate_cluster_exchange(4, 8, seed=seed, slow=seed % 4, slow_factor=30, nslots=1)
        except ProtocolViolation:
            caught += 1
    assert caught >= 5
