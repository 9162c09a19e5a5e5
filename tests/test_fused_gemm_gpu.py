"""Layer-boundary fusion (row-parallel GEMM -> all-reduce + residual + RMSNorm -> column-parallel GEMM)
with every rank emulated on one GPU.

`gemm_push` runs all ranks' GEMMs in one launch and pushes the partial outputs into the landing
buffers; `ar_norm_gemm` (one launch, all ranks) waits for them, so the two launches never wait on
each other. Oracle: fp32 GEMMs, fp32 sum + residual + RMSNorm, fp32 second GEMM; relative error
max|out - ref| / max|ref| <= 2^-5 (the acceptance rule of the fused op,
exp/M17_epoch_ab/bench_ab.py:160-164).
"""
import pytest
import torch

from comm_opt_b200.ops.reference import TOL, rel_err
from comm_opt_b200.parallel import TPCommunicator

pytestmark = pytest.mark.gpu


def reference(x, w1, res0, gamma, w2, eps):
    """x [W, M, K1], w1 [W, H, K1], res0 [M, H], w2 [W, N2, H] -> (h [M, H], out [W, M, N2])."""
    y = sum(x[r].float() @ w1[r].float().t() for r in range(x.shape[0]))
    h = res0.float() + y
    n = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()
    return h, torch.stack([n @ w2[r].float().t() for r in range(x.shape[0])])


def layer_boundary(comm, x, w1, res, gamma, w2, eps, splits1=0, splits2=0):
    comm.gemm_push(x, w1, splits=splits1)
    return comm.ar_norm_gemm(res, gamma, w2, eps, splits=splits2)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("M", [1, 5, 16, 40])
def test_layer_boundary_emulated(cuda, world, M):
    K1, H, N2, eps = 512, 1024, 384, 1e-5
    comm = TPCommunicator(emulate_world=world, device=cuda, dtype=torch.bfloat16, max_rows=64, max_hidden=H)
    g = torch.Generator(device=cuda).manual_seed(M * 10 + world)
    w1 = (0.02 * torch.randn(world, H, K1, generator=g, device=cuda)).bfloat16()
    w2 = (0.02 * torch.randn(world, N2, H, generator=g, device=cuda)).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).bfloat16()
    res0 = torch.randn(M, H, generator=g, device=cuda).bfloat16()
    res = res0.unsqueeze(0).repeat(world, 1, 1).contiguous()
    for it in range(3):  # consecutive calls alternate landing slots and reuse the pieces' flags
        x = torch.randn(world, M, K1, generator=g, device=cuda).bfloat16()
        before = res[0].clone()
        out = layer_boundary(comm, x, w1, res, gamma, w2, eps, splits1=2, splits2=2)
        torch.cuda.synchronize()
        comm.check()
        h_ref, out_ref = reference(x, w1, before, gamma, w2, eps)
        for r in range(world):
            assert rel_err(res[r], h_ref) <= TOL, (it, r, rel_err(res[r], h_ref))
            assert rel_err(out[r], out_ref[r]) <= TOL, (it, r, rel_err(out[r], out_ref[r]))
        for r in range(1, world):
            assert torch.equal(res[r], res[0])
    assert comm.epochs() == [3] * world


def test_layer_boundary_interleaved_with_fused_ar(cuda):
    """The fused GEMMs and the standalone fused op share the epoch and the landing slots."""
    world, M, K1, H, N2, eps = 4, 8, 256, 2048, 256, 1e-6
    comm = TPCommunicator(emulate_world=world, device=cuda, dtype=torch.bfloat16, max_rows=16, max_hidden=H)
    g = torch.Generator(device=cuda).manual_seed(3)
    w1 = (0.05 * torch.randn(world, H, K1, generator=g, device=cuda)).bfloat16()
    w2 = (0.05 * torch.randn(world, N2, H, generator=g, device=cuda)).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).bfloat16()
    res = torch.randn(M, H, generator=g, device=cuda).bfloat16().unsqueeze(0).repeat(world, 1, 1).contiguous()
    for it in range(4):
        if it % 2:
            xs = torch.randn(world, M, H, generator=g, device=cuda).bfloat16()
            before = res[0].clone()
            out = torch.empty_like(xs)
            comm.fused_allreduce_add_rmsnorm(xs, res, gamma, eps, out=out, variant="lamport_1s")
            torch.cuda.synchronize()
            h_ref = before.float() + xs.float().sum(0)
            assert rel_err(res[0], h_ref) <= TOL
        else:
            x = torch.randn(world, M, K1, generator=g, device=cuda).bfloat16()
            before = res[0].clone()
            out = layer_boundary(comm, x, w1, res, gamma, w2, eps)
            torch.cuda.synchronize()
            h_ref, out_ref = reference(x, w1, before, gamma, w2, eps)
            assert rel_err(res[0], h_ref) <= TOL and rel_err(out[1], out_ref[1]) <= TOL, it
    comm.check()
    assert comm.epochs() == [4] * world


@pytest.mark.parametrize("M", [8, 32])
def test_layer_boundary_70b_tp8_shapes(cuda, M):
    """Llama-70B TP=8 shapes, 2 emulated ranks: down_proj [M, 3584] x [8192, 3584]^T ->
    AR + residual + RMSNorm -> QKV [M, 8192] x [1280, 8192]^T (default split plans)."""
    world, K1, H, N2, eps = 2, 3584, 8192, 1280, 1e-5
    comm = TPCommunicator(emulate_world=world, device=cuda, dtype=torch.bfloat16, max_rows=M, max_hidden=H)
    g = torch.Generator(device=cuda).manual_seed(M)
    w1 = (0.02 * torch.randn(world, H, K1, generator=g, device=cuda)).bfloat16()
    w2 = (0.02 * torch.randn(world, N2, H, generator=g, device=cuda)).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).bfloat16()
    res0 = torch.randn(M, H, generator=g, device=cuda).bfloat16()
    res = res0.unsqueeze(0).repeat(world, 1, 1).contiguous()
    x = torch.randn(world, M, K1, generator=g, device=cuda).bfloat16()
    out = layer_boundary(comm, x, w1, res, gamma, w2, eps)
    torch.cuda.synchronize()
    comm.check()
    h_ref, out_ref = reference(x, w1, res0, gamma, w2, eps)
    for r in range(world):
        assert rel_err(res[r], h_ref) <= TOL
        assert rel_err(out[r], out_ref[r]) <= TOL


@pytest.mark.parametrize("world", [2, 4])
def test_layer_boundary_many_tiles(cuda, world):
    """More output tiles than resident CTAs: ar_norm_gemm drops split-K and loops over tiles per CTA
    (double-buffered accumulators), as for gate_up / the LM head at TP <= 4."""
    M, K1, H, N2, eps = 8, 256, 1024, 24576, 1e-5  # 192 output tiles > resident CTAs per rank
    comm = TPCommunicator(emulate_world=world, device=cuda, dtype=torch.bfloat16, max_rows=16, max_hidden=H)
    g = torch.Generator(device=cuda).manual_seed(world)
    w1 = (0.05 * torch.randn(world, H, K1, generator=g, device=cuda)).bfloat16()
    w2 = (0.05 * torch.randn(world, N2, H, generator=g, device=cuda)).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).bfloat16()
    res = torch.randn(M, H, generator=g, device=cuda).bfloat16().unsqueeze(0).repeat(world, 1, 1).contiguous()
    for it in range(2):
        x = torch.randn(world, M, K1, generator=g, device=cuda).bfloat16()
        before = res[0].clone()
        out = layer_boundary(comm, x, w1, res, gamma, w2, eps)
        torch.cuda.synchronize()
        comm.check()
        kind, plan = comm.last_fused_gemm
        assert plan[2] == 1 and plan[4] < plan[1], plan  # no split-K, fewer CTAs than tiles
        h_ref, out_ref = reference(x, w1, before, gamma, w2, eps)
        for r in range(world):
            assert rel_err(res[r], h_ref) <= TOL
            assert rel_err(out[r], out_ref[r]) <= TOL, (it, r, rel_err(out[r], out_ref[r]))


def test_layer_boundary_split16(cuda):
    """Split-K over a 16-CTA (non-portable) cluster, the plan for narrow outputs such as QKV at TP=8."""
    world, M, K1, H, N2, eps = 2, 8, 512, 2048, 640, 1e-5
    comm = TPCommunicator(emulate_world=world, device=cuda, dtype=torch.bfloat16, max_rows=8, max_hidden=H)
    g = torch.Generator(device=cuda).manual_seed(16)
    w1 = (0.05 * torch.randn(world, H, K1, generator=g, device=cuda)).bfloat16()
    w2 = (0.05 * torch.randn(world, N2, H, generator=g, device=cuda)).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).bfloat16()
    res0 = torch.randn(M, H, generator=g, device=cuda).bfloat16()
    res = res0.unsqueeze(0).repeat(world, 1, 1).contiguous()
    x = torch.randn(world, M, K1, generator=g, device=cuda).bfloat16()
    out = layer_boundary(comm, x, w1, res, gamma, w2, eps, splits2=16)
    torch.cuda.synchronize()
    comm.check()
    assert comm.last_fused_gemm[1][2] == 16
    h_ref, out_ref = reference(x, w1, res0, gamma, w2, eps)
    for r in range(world):
        assert rel_err(res[r], h_ref) <= TOL
        assert rel_err(out[r], out_ref[r]) <= TOL


@pytest.mark.parametrize("world", [2, 8])
def test_layer_boundary_swiglu_epilogue(cuda, world):
    """down_proj push -> AR + residual + RMSNorm -> gate_up with SiLU(gate) * up in the epilogue."""
    M, K1, H, I, eps = 8, 512, 1024, 448, 1e-5  # I = 7 tiles of 64
    comm = TPCommunicator(emulate_world=world, device=cuda, dtype=torch.bfloat16, max_rows=8, max_hidden=H)
    g = torch.Generator(device=cuda).manual_seed(world + 40)
    w1 = (0.05 * torch.randn(world, H, K1, generator=g, device=cuda)).bfloat16()
    wgu = (0.05 * torch.randn(world, 2 * I, H, generator=g, device=cuda)).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).bfloat16()
    res0 = torch.randn(M, H, generator=g, device=cuda).bfloat16()
    res = res0.unsqueeze(0).repeat(world, 1, 1).contiguous()
    x = torch.randn(world, M, K1, generator=g, device=cuda).bfloat16()
    comm.gemm_push(x, w1)
    act = comm.ar_norm_gemm(res, gamma, TPCommunicator.interleave_gate_up(wgu), eps, epilogue="swiglu")
    torch.cuda.synchronize()
    comm.check()
    assert act.shape == (world, M, I) and 2 <= comm.last_fused_gemm[1][2] <= 8
    h_ref, gu_ref = reference(x, w1, res0, gamma, wgu, eps)
    for r in range(world):
        gg, uu = gu_ref[r].bfloat16().float().chunk(2, -1)
        ref = torch.nn.functional.silu(gg) * uu
        assert rel_err(res[r], h_ref) <= TOL
        assert rel_err(act[r], ref) <= TOL, (r, rel_err(act[r], ref))


@pytest.mark.parametrize("world", [2, 4])
def test_layer_boundary_rope_kv_epilogue(cuda, world):
    """AR + RMSNorm -> QKV with RoPE on q/k and the paged KV append in the epilogue."""
    from comm_opt_b200.ops.reference import rope_tables

    M, K1, H, nq, nkv, D, bs, eps = 6, 256, 1024, 4, 2, 128, 16, 1e-5
    N = (nq + 2 * nkv) * D
    comm = TPCommunicator(emulate_world=world, device=cuda, dtype=torch.bfloat16, max_rows=8, max_hidden=H)
    g = torch.Generator(device=cuda).manual_seed(world + 50)
    w1 = (0.05 * torch.randn(world, H, K1, generator=g, device=cuda)).bfloat16()
    wqkv = (0.05 * torch.randn(world, N, H, generator=g, device=cuda)).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).bfloat16()
    res0 = torch.randn(M, H, generator=g, device=cuda).bfloat16()
    res = res0.unsqueeze(0).repeat(world, 1, 1).contiguous()
    x = torch.randn(world, M, K1, generator=g, device=cuda).bfloat16()
    maxb, nblocks = 4, 40
    pos = torch.tensor([0, 5, 16, 17, 40, 63], dtype=torch.int32, device=cuda)
    bt = torch.randperm(nblocks, generator=torch.Generator().manual_seed(2))[:M * maxb].view(M, maxb)
    bt = bt.to(torch.int32).to(cuda)
    kc = torch.zeros(world, nblocks, nkv, bs, D, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    cos, sin = rope_tables(128, D, 5e5, cuda)
    comm.gemm_push(x, w1)
    q = comm.ar_norm_gemm(res, gamma, wqkv, eps, epilogue="rope_kv",
                          rope=dict(positions=pos, cos=cos, sin=sin, block_tables=bt, k_cache=kc, v_cache=vc,
                                    nq=nq, nkv=nkv))
    torch.cuda.synchronize()
    comm.check()
    h_ref, z_ref = reference(x, w1, res0, gamma, wqkv, eps)
    half = D // 2
    c, s = cos[pos.long()][:, None, :], sin[pos.long()][:, None, :]  # [M, 1, 64]: row b at position pos[b]

    def rot(t):  # t [M, heads, D]
        return torch.cat([t[..., :half] * c - t[..., half:] * s, t[..., half:] * c + t[..., :half] * s], -1)

    for r in range(world):
        z = z_ref[r].bfloat16().float().view(M, nq + 2 * nkv, D)
        qref, kref, vref = rot(z[:, :nq]), rot(z[:, nq:nq + nkv]), z[:, nq + nkv:]
        assert rel_err(q[r].view(M, nq, D), qref) <= TOL
        for b in range(M):
            blk, off = int(bt[b, int(pos[b]) // bs]), int(pos[b]) % bs
            assert rel_err(kc[r, blk, :, off], kref[b]) <= TOL, (r, b)
            assert rel_err(vc[r, blk, :, off], vref[b]) <= TOL, (r, b)


@pytest.mark.parametrize("world,M,K1,H,N2,splits2", [(2, 8, 3584, 8192, 1280, 0), (4, 5, 512, 1024, 24576, 0),
                                                    (2, 8, 512, 2048, 640, 16), (2, 3, 256, 1024, 296, 0)])
def test_layer_boundary_packed_weights(cuda, world, M, K1, H, N2, splits2):
    """Both fused GEMMs on packed (bulk-load) weights give the bits of the row-major launches: 70B TP=8
    shapes, many tiles per CTA, a 16-CTA cluster, and an output width that is not a multiple of 128."""
    from comm_opt_b200.models.gemm import pack_weight

    eps = 1e-5
    g = torch.Generator(device=cuda).manual_seed(M + N2)
    w1 = (0.02 * torch.randn(world, H, K1, generator=g, device=cuda)).bfloat16()
    w2 = (0.02 * torch.randn(world, N2, H, generator=g, device=cuda)).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device=cuda)).bfloat16()
    res0 = torch.randn(M, H, generator=g, device=cuda).bfloat16()
    x = torch.randn(world, M, K1, generator=g, device=cuda).bfloat16()
    outs = []
    for packed in (False, True):
        comm = TPCommunicator(emulate_world=world, device=cuda, dtype=torch.bfloat16, max_rows=16, max_hidden=H)
        res = res0.unsqueeze(0).repeat(world, 1, 1).contiguous()
        a, b = (pack_weight(w1), pack_weight(w2)) if packed else (w1, w2)
        out = layer_boundary(comm, x, a, res, gamma, b, eps, splits2=splits2)
        torch.cuda.synchronize()
        comm.check()
        outs.append((res, out))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    h_ref, out_ref = reference(x, w1, res0, gamma, w2, eps)
    for r in range(world):
        assert rel_err(outs[1][0][r], h_ref) <= TOL
        assert rel_err(outs[1][1][r], out_ref[r]) <= TOL
