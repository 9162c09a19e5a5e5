"""Single-GPU tier of the fused all-reduce + residual + RMSNorm: all ranks emulated in one launch.

Every rank's heap is a separate region of this GPU and one kernel launch runs every rank (grid.y =
world), so the cross-rank protocol (Lamport landing, flag barriers, epochs) executes for real
without separate launches that wait on one another. Oracle: fp32 sum + residual + RMSNorm,
relative error <= 2^-5 (the reference's criterion, exp/M17_epoch_ab/bench_ab.py:160-164); fp32
inputs are held to 1e-5.
"""
import os
import random

import pytest
import torch

from comm_opt_b200.ops.reference import TOL, fused_allreduce_add_rmsnorm_ref, rel_err
from comm_opt_b200.parallel import TPCommTimeout, TPCommunicator

pytestmark = pytest.mark.gpu

EMU_VARIANTS = ["lamport_1s", "lamport_2s", "pull_1s", "pull_2s"]

# Kernels once written without a GPU at hand (the cluster row-sum exchange form): they have passed on B200
# and run with every other test; the marker stays as the place to gate the next such kernel.
experimental = pytest.mark.skipif(os.environ.get("COB_SKIP_EXPERIMENTAL") == "1",
                                  reason="COB_SKIP_EXPERIMENTAL=1")


def make_inputs(world, rows, hidden, dtype, dev, seed=0, scale=1.0):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = (scale * torch.randn(world, rows, hidden, generator=g, device=dev)).to(dtype)
    res0 = torch.randn(rows, hidden, generator=g, device=dev).to(dtype)
    gamma = (1 + 0.1 * torch.randn(hidden, generator=g, device=dev)).to(dtype)
    return x, res0, gamma


def check(comm, x, res0, gamma, eps, variant, **kw):
    world = x.shape[0]
    res = res0.unsqueeze(0).repeat(world, 1, 1).contiguous()
    out = torch.empty_like(x)
    comm.fused_allreduce_add_rmsnorm(x, res, gamma, eps, out=out, variant=variant, **kw)
    torch.cuda.synchronize()
    comm.check()
    ref_out, ref_h = fused_allreduce_add_rmsnorm_ref(list(x), res0, gamma, eps)
    tol = 1e-5 if x.dtype == torch.float32 else TOL
    for r in range(world):
        assert rel_err(out[r], ref_out) <= tol, (variant, r, rel_err(out[r], ref_out))
        assert rel_err(res[r], ref_h) <= tol, (variant, r, rel_err(res[r], ref_h))
    # every rank holds bitwise the same result (same summation order everywhere)
    for r in range(1, world):
        assert torch.equal(out[r], out[0]) and torch.equal(res[r], res[0])
    return out, res


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("variant", EMU_VARIANTS)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_variants_emulated(cuda, world, variant, dtype):
    comm = TPCommunicator(emulate_world=world, device=cuda, dtype=dtype, max_rows=64, max_hidden=8192)
    for rows, hidden in [(1, 8192), (3, 4096), (17, 2048), (64, 1024)]:
        x, res0, gamma = make_inputs(world, rows, hidden, dtype, cuda, seed=rows)
        check(comm, x, res0, gamma, 1e-6, variant)
    assert comm.epochs() == [4] * world


@pytest.mark.parametrize("variant", EMU_VARIANTS)
def test_plain_allreduce_emulated(cuda, variant):
    comm = TPCommunicator(emulate_world=4, device=cuda, dtype=torch.bfloat16, max_rows=32, max_hidden=4096)
    x = torch.randn(4, 5, 4096, device=cuda).to(torch.bfloat16)
    out = comm.all_reduce(x, variant=variant)
    torch.cuda.synchronize()
    comm.check()
    ref = x.float().sum(0)
    for r in range(4):
        assert rel_err(out[r], ref) <= TOL


def test_geometry_overrides_and_clusters(cuda):
    comm = TPCommunicator(emulate_world=2, device=cuda, dtype=torch.bfloat16, max_rows=16, max_hidden=8192)
    x, res0, gamma = make_inputs(2, 4, 8192, torch.bfloat16, cuda)
    for cluster in (1, 2, 4, 8):
        check(comm, x, res0, gamma, 1e-5, "lamport_1s", cluster=cluster, blocks=4 * cluster)
        assert comm.last_choice.cluster == cluster
    for blocks in (1, 3, 16):
        check(comm, x, res0, gamma, 1e-5, "lamport_2s", blocks=blocks, threads=256)
        check(comm, x, res0, gamma, 1e-5, "pull_2s", blocks=blocks)


def test_negative_zero_inputs(cuda):
    """Senders map -0 to +0 so the Lamport sentinel can never be sent as data."""
    comm = TPCommunicator(emulate_world=4, device=cuda, dtype=torch.bfloat16, max_rows=8, max_hidden=1024)
    x = torch.full((4, 2, 1024), -0.0, device=cuda, dtype=torch.bfloat16)
    x[:, 1] = 1.0
    for v in EMU_VARIANTS:
        out = comm.all_reduce(x, variant=v)
        torch.cuda.synchronize()
        comm.check()
        assert torch.all(out[:, 0] == 0) and torch.all(out[:, 1] == 4)


@pytest.mark.parametrize("mode", ["eager", "graph"])
def test_interleaving(cuda, mode):
    """Port of the reference's interleaving test (exp/M16_epoch_fix/test_interleave.py): 60 calls,
    random token counts, block counts and variants, no state reset; graph mode keeps one CUDA graph
    per combination and replays them in random order."""
    interleave(cuda, mode, EMU_VARIANTS)


def interleave(cuda, mode, variants):
    world, H, dtype = 8, 5120, torch.bfloat16
    comm = TPCommunicator(emulate_world=world, device=cuda, dtype=dtype, max_rows=128, max_hidden=H)
    rng = random.Random(0)
    tokens, blocks = [1, 3, 8, 13, 40, 64, 128], [1, 2, 4, 8, 16]
    seq = [(rng.choice(tokens), rng.choice(blocks), rng.choice(variants)) for _ in range(60)]
    g = torch.Generator(device=cuda).manual_seed(7)
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).to(dtype)
    graphs = {}
    if mode == "graph":
        for key in sorted(set(seq)):
            nt, nb, v = key
            x = torch.zeros(world, nt, H, device=cuda, dtype=dtype)
            res = torch.zeros(world, nt, H, device=cuda, dtype=dtype)
            out = torch.empty_like(x)
            # warm the variant (also advances the epoch on every rank alike)
            comm.fused_allreduce_add_rmsnorm(x, res, gamma, 1e-6, out=out, variant=v, blocks=nb)
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                comm.fused_allreduce_add_rmsnorm(x, res, gamma, 1e-6, out=out, variant=v, blocks=nb)
            graphs[key] = (gr, x, res, out)
        torch.cuda.synchronize()
    for i, (nt, nb, v) in enumerate(seq):
        x, res0, _ = make_inputs(world, nt, H, dtype, cuda, seed=1000 + i)
        if mode == "eager":
            res = res0.unsqueeze(0).repeat(world, 1, 1).contiguous()
            out = torch.empty_like(x)
            comm.fused_allreduce_add_rmsnorm(x, res, gamma, 1e-6, out=out, variant=v, blocks=nb)
        else:
            gr, xg, res, out = graphs[(nt, nb, v)]
            xg.copy_(x)
            res.copy_(res0.unsqueeze(0).expand_as(res))
            gr.replay()
        torch.cuda.synchronize()
        ref_out, ref_h = fused_allreduce_add_rmsnorm_ref(list(x), res0, gamma, 1e-6)
        for r in range(world):
            assert rel_err(out[r], ref_out) <= TOL, (i, nt, nb, v, r)
            assert rel_err(res[r], ref_h) <= TOL, (i, nt, nb, v, r)
    comm.check()
    del graphs


def test_bounded_wait_times_out_without_peer(cuda):
    """Rank 0 of a 2-rank communicator runs alone (rank 1's heap exists, its kernel never runs): every
    wait gives up after the timeout, the error word is set, the host raises, and reset() recovers."""
    comm = TPCommunicator(emulate_world=2, device=cuda, dtype=torch.bfloat16, max_rows=4, max_hidden=1024,
                          timeout_ms=50)
    from comm_opt_b200._ext import native

    x = torch.randn(2, 1024, device=cuda).to(torch.bfloat16)
    out = torch.empty_like(x)
    for variant in (1, 2, 5, 6):
        rc = native().fused_ar(comm.heap.bases, 0, comm._layout_list, x, x, x[0], out, 0, 2, 1024, 1e-6, variant, 0,
                               0, 0, 0, 0, 0, comm.timeout_ns, 0, 0, 0, False)
        assert rc[0] == 0
        torch.cuda.synchronize()
        with pytest.raises(TPCommTimeout):
            comm.check()
        comm.reset()
        assert all(s["error"] == 0 for s in comm.error_state())
    # the communicator still works after the reset
    xe, res0, gamma = make_inputs(2, 2, 1024, torch.bfloat16, cuda)
    check(comm, xe, res0, gamma, 1e-6, "lamport_1s")


def test_allgather_u32_emulated(cuda):
    comm = TPCommunicator(emulate_world=4, device=cuda, dtype=torch.bfloat16, max_rows=4, max_hidden=1024)
    for it in range(3):
        inp = torch.arange(4 * 10, device=cuda, dtype=torch.int32).view(4, 10) * (it + 1)
        out = comm.all_gather_u32(inp)
        torch.cuda.synchronize()
        comm.check()
        for r in range(4):
            assert torch.equal(out[r], inp)


def test_phase_stamps_and_overhead(cuda):
    """Stamped calls record ordered phase times for every block; outputs unchanged."""
    comm = TPCommunicator(emulate_world=4, device=cuda, dtype=torch.bfloat16, max_rows=16, max_hidden=8192)
    x, res0, gamma = make_inputs(4, 8, 8192, torch.bfloat16, cuda)
    for v in EMU_VARIANTS:
        comm.disable_stamps()
        out_plain, _ = check(comm, x, res0, gamma, 1e-6, v)
        comm.enable_stamps(cap=64)
        out_st, _ = check(comm, x, res0, gamma, 1e-6, v)
        assert torch.equal(out_plain, out_st)
        e = comm.epochs()[0]
        blocks = comm.last_choice.blocks
        summ = comm.stamp_summary([e], blocks)
        for r in range(4):
            ph = summ[r]
            assert 0 <= ph["sent"] <= ph["done"] and ph["received"] <= ph["done"] + 1e-3, (v, ph)
    comm.disable_stamps()


# ------------------------------------------------------------------ lamport_1sx (experimental)
@experimental
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_lamport_1sx_matches_lamport_1s(cuda, world, dtype):
    """The cluster row-sum exchange changes only how the partial sums meet: outputs and residuals
    equal lamport_1s bit for bit, for every cluster size and for rows spread over several CTAs."""
    comm = TPCommunicator(emulate_world=world, device=cuda, dtype=dtype, max_rows=64, max_hidden=8192)
    budget = 148 // world
    for rows, hidden in [(1, 8192), (3, 4096), (17, 2048), (64, 1024)]:
        x, res0, gamma = make_inputs(world, rows, hidden, dtype, cuda, seed=rows)
        for cluster in (1, 2, 4, 8):
            blocks = cluster * max(1, min(rows, budget // cluster, 4))
            out_a, res_a = check(comm, x, res0, gamma, 1e-6, "lamport_1s", cluster=cluster, blocks=blocks)
            out_b, res_b = check(comm, x, res0, gamma, 1e-6, "lamport_1sx", cluster=cluster, blocks=blocks)
            assert comm.last_choice.cluster == cluster
            assert torch.equal(out_a, out_b) and torch.equal(res_a, res_b), (rows, hidden, cluster)


@experimental
@pytest.mark.parametrize("mode", ["eager", "graph"])
def test_lamport_1sx_interleaving(cuda, mode):
    interleave(cuda, mode, ["lamport_1sx", "lamport_1s", "lamport_2s", "lamport_1sx"])


@experimental
def test_lamport_1sx_times_out_without_peer(cuda):
    comm = TPCommunicator(emulate_world=2, device=cuda, dtype=torch.bfloat16, max_rows=4, max_hidden=1024,
                          timeout_ms=50)
    from comm_opt_b200._ext import native

    x = torch.randn(2, 1024, device=cuda).to(torch.bfloat16)
    out = torch.empty_like(x)
    for cluster in (1, 4):
        rc = native().fused_ar(comm.heap.bases, 0, comm._layout_list, x, x, x[0], out, 0, 2, 1024, 1e-6, 7, 0,
                               0, cluster, 0, 0, 1, comm.timeout_ns, 0, 0, 0, False)
        assert rc[0] == 0
        torch.cuda.synchronize()
        with pytest.raises(TPCommTimeout):
            comm.check()
        comm.reset()
    xe, res0, gamma = make_inputs(2, 2, 1024, torch.bfloat16, cuda)
    check(comm, xe, res0, gamma, 1e-6, "lamport_1sx")
