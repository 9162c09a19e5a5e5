"""tcgen05 decode GEMM against a plain fp32 PyTorch matmul."""
import pytest
import torch

from comm_opt_b200.models.gemm import gemm, gemm_error_word
from comm_opt_b200.ops.reference import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (8, 1280, 8192), (3, 300, 200), (16, 8192, 1024),
                                   (32, 7168, 1024), (64, 1024, 3584), (128, 16032, 512), (200, 512, 4096),
                                   (256, 256, 256), (300, 384, 128)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemm_matches_fp32(cuda, M, N, K, dtype):
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N)
    x = torch.randn(M, K, device=cuda, generator=g).to(dtype)
    w = (0.05 * torch.randn(N, K, device=cuda, generator=g)).to(dtype)
    ref = x.float() @ w.float().t()
    y = gemm(x, w)
    torch.cuda.synchronize()
    assert int(gemm_error_word(cuda)) == 0
    assert rel_err(y, ref) <= 2 ** -7, rel_err(y, ref)


@pytest.mark.parametrize("ctas", [1, 3, 7, 37, 148, 500])
def test_gemm_stream_k_partitions_deterministic(cuda, ctas):
    """Any CTA count (tiles split between many CTAs, CTAs spanning several tiles) gives the same
    bits on repeated calls and matches fp32."""
    x = torch.randn(8, 4096, device=cuda).to(torch.bfloat16)
    w = (0.05 * torch.randn(640, 4096, device=cuda)).to(torch.bfloat16)
    y1 = gemm(x, w, ctas=ctas)
    y2 = gemm(x, w, ctas=ctas)
    torch.cuda.synchronize()
    assert int(gemm_error_word(cuda)) == 0
    assert torch.equal(y1, y2)
    assert rel_err(y1, x.float() @ w.float().t()) <= 2 ** -7


def test_gemm_into_strided_output_and_graph(cuda):
    x = torch.randn(4, 1024, device=cuda).to(torch.bfloat16)
    w = (0.05 * torch.randn(2048, 1024, device=cuda)).to(torch.bfloat16)
    big = torch.zeros(4, 4096, device=cuda, dtype=torch.bfloat16)
    out = big[:, 1024:3072]
    gemm(x, w, out)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gemm(x, w, out)
    x.mul_(2)
    g.replay()
    torch.cuda.synchronize()
    assert rel_err(out, x.float() @ w.float().t()) <= 2 ** -7
    assert torch.all(big[:, :1024] == 0) and torch.all(big[:, 3072:] == 0)


@pytest.mark.parametrize("splits", [2, 3, 5, 8, 12, 16])
@pytest.mark.parametrize("small", [False, True])
def test_gemm_cluster_split_k(cuda, splits, small):
    """Cluster split-K schedule (partial rows pushed to their owner CTA over distributed shared memory)
    against fp32, deterministic across calls; 12 and 16 splits are non-portable clusters (half ring)."""
    if splits > 8 and not small:
        pytest.skip("clusters above 8 CTAs run with the half ring (two CTAs per SM)")
    for M, N, K in [(1, 1280, 8192), (8, 300, 1000), (64, 8192, 1024)]:
        x = torch.randn(M, K, device=cuda).to(torch.bfloat16)
        w = (0.05 * torch.randn(N, K, device=cuda)).to(torch.bfloat16)
        y1 = gemm(x, w, cluster_splits=splits, small_smem=small)
        y2 = gemm(x, w, cluster_splits=splits, small_smem=small)
        torch.cuda.synchronize()
        assert int(gemm_error_word(cuda)) == 0
        assert torch.equal(y1, y2)
        assert rel_err(y1, x.float() @ w.float().t()) <= 2 ** -7, (M, N, K, rel_err(y1, x.float() @ w.float().t()))


def test_gemm_tuner_picks_valid_config(cuda):
    from comm_opt_b200.models.gemm import Linear

    w = (0.05 * torch.randn(1280, 8192, device=cuda)).to(torch.bfloat16)
    lin = Linear(w)
    cfg = lin.tune(8)
    assert isinstance(cfg, dict)
    x = torch.randn(8, 8192, device=cuda).to(torch.bfloat16)
    assert rel_err(lin(x), x.float() @ w.float().t()) <= 2 ** -7


@pytest.mark.parametrize("tiles", [4, 16, 64])
def test_gemm_l2_prefetch_same_bits(cuda, tiles):
    """Prefetching weight tiles into L2 is only a hint: stream-K and cluster split-K results are bitwise
    those without it (partial last tile, M not a multiple of the batch tile, K beyond the ring)."""
    from comm_opt_b200.ops.kernels import set_l2_prefetch

    x = torch.randn(5, 8192, device=cuda).to(torch.bfloat16)
    w = (0.05 * torch.randn(1000, 8192, device=cuda)).to(torch.bfloat16)
    base = [gemm(x, w), gemm(x, w, cluster_splits=4)]
    old = set_l2_prefetch(tiles)
    try:
        got = [gemm(x, w), gemm(x, w, cluster_splits=4)]
    finally:
        set_l2_prefetch(old)
    torch.cuda.synchronize()
    assert int(gemm_error_word(cuda)) == 0
    assert all(torch.equal(a, b) for a, b in zip(base, got))


@pytest.mark.parametrize("M,N,K", [(1, 128, 64), (8, 1280, 8192), (3, 300, 192), (16, 8192, 1024),
                                   (64, 1024, 3584), (128, 16032, 512), (200, 512, 4096)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("sched", [dict(), dict(small_smem=True, pdl=True), dict(cluster_splits=4),
                                   dict(ctas=5)])
def test_packed_weights_match_row_major(cuda, M, N, K, dtype, sched):
    """The packed (bulk-load) weight layout gives the bits of the row-major launch of the same schedule."""
    from comm_opt_b200.models.gemm import pack_weight

    if sched.get("cluster_splits") and M > 64:
        pytest.skip("cluster split-K is for M <= 64")
    g = torch.Generator(device=cuda).manual_seed(M * 5 + N + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(dtype)
    w = (0.05 * torch.randn(N, K, device=cuda, generator=g)).to(dtype)
    pw = pack_weight(w)
    assert torch.equal(pw.dense(), w)
    y_rm = gemm(x, w, **sched)
    y_pk = gemm(x, pw, **sched)
    torch.cuda.synchronize()
    assert int(gemm_error_word(cuda)) == 0
    assert torch.equal(y_rm, y_pk)
    assert rel_err(y_pk, x.float() @ w.float().t()) <= 2 ** -7


@pytest.mark.parametrize("M,I,K", [(1, 64, 64), (8, 3584, 8192), (5, 192, 1024), (16, 7168, 1024), (64, 128, 512)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("splits,small", [(2, False), (4, True), (8, True), (16, True)])
@pytest.mark.parametrize("packed", [True, False])
def test_gemm_swiglu_epilogue(cuda, M, I, K, dtype, splits, small, packed):
    """GEMM with the SwiGLU epilogue (gate/up rows interleaved by 64): silu(gate) * up of the fp32
    projection within bf16/fp16 tolerance, and the same bits as the plain launch of the same schedule
    followed by the SiLU * up kernel on its interleaved output."""
    from comm_opt_b200.models.gemm import interleave_rows, pack_weight, swiglu_splits
    from comm_opt_b200.ops import kernels as K_

    if not swiglu_splits(K, splits):
        pytest.skip("split count the epilogue does not accept for this K")
    g = torch.Generator(device=cuda).manual_seed(M * 3 + I + K + splits)
    x = torch.randn(M, K, device=cuda, generator=g).to(dtype)
    w = (0.05 * torch.randn(2 * I, K, device=cuda, generator=g)).to(dtype)
    wi = pack_weight(w, interleave=64) if packed else interleave_rows(w, 64)
    if packed:
        assert torch.equal(wi.dense(), w)
    sched = dict(cluster_splits=splits, small_smem=small, pdl=small)
    act = gemm(x, wi, swiglu=True, **sched)
    plain = gemm(x, wi, **sched)
    torch.cuda.synchronize()
    assert int(gemm_error_word(cuda)) == 0
    assert act.shape == (M, I)
    assert torch.equal(act, K_.silu_mul(plain, interleave=64))
    gu = x.float() @ w.float().t()
    ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    assert rel_err(act, ref) <= 2 ** -6, rel_err(act, ref)


@pytest.mark.parametrize("M,I,K", [(1, 64, 1024), (8, 3584, 8192), (5, 192, 4096), (16, 1024, 2048)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("sched", [dict(), dict(small_smem=True, pdl=True), dict(ctas=5), dict(ctas=7),
                                   dict(ctas="tiles")])
def test_gemm_swiglu_epilogue_stream_k(cuda, M, I, K, dtype, sched):
    """Stream-K with the SwiGLU epilogue (M <= 16): whole tiles and tiles split between CTAs (their last
    contributor finishes them) give the bits of the plain launch of the same schedule followed by the
    SiLU * up kernel, and silu(gate) * up of the fp32 projection within tolerance."""
    from comm_opt_b200.models.gemm import pack_weight
    from comm_opt_b200.ops import kernels as K_

    g = torch.Generator(device=cuda).manual_seed(M * 7 + I + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(dtype)
    w = (0.05 * torch.randn(2 * I, K, device=cuda, generator=g)).to(dtype)
    wi = pack_weight(w, interleave=64)
    sched = dict(sched)
    if sched.get("ctas") == "tiles":
        sched["ctas"] = (2 * I) // 128  # one CTA per output tile: whole tiles only
    act = gemm(x, wi, swiglu=True, **sched)
    plain = gemm(x, wi, **sched)
    torch.cuda.synchronize()
    assert int(gemm_error_word(cuda)) == 0
    assert torch.equal(act, K_.silu_mul(plain, interleave=64))
    gu = x.float() @ w.float().t()
    ref = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    assert rel_err(act, ref) <= 2 ** -6, rel_err(act, ref)


def test_gemm_swiglu_rejects_other_schedules(cuda):
    """The SwiGLU epilogue is refused (not silently wrong) for stream-K beyond 16 rows and for split counts
    that do not pair every gate row with its up row inside one CTA."""
    x = torch.randn(8, 1024, device=cuda).bfloat16()
    w = torch.randn(256, 1024, device=cuda).bfloat16()
    with pytest.raises(ValueError):
        gemm(torch.randn(32, 1024, device=cuda).bfloat16(), w, swiglu=True)
    with pytest.raises(RuntimeError):
        gemm(x, w, cluster_splits=3, swiglu=True)  # 3 CTAs per tile
    with pytest.raises(RuntimeError):
        gemm(x, torch.randn(192, 1024, device=cuda).bfloat16(), cluster_splits=2, swiglu=True)  # N % 128


def test_gate_up_linear_tuned_and_fallback(cuda):
    """GateUpLinear: the tuned SwiGLU-epilogue launch and the two-kernel fallback give the same bits."""
    from comm_opt_b200.models.gemm import GateUpLinear, pack_weight

    g = torch.Generator(device=cuda).manual_seed(11)
    x = torch.randn(8, 2048, device=cuda, generator=g).bfloat16()
    w = (0.05 * torch.randn(2 * 1024, 2048, device=cuda, generator=g)).bfloat16()
    lin = GateUpLinear(pack_weight(w, interleave=64))
    lin.tune(8)  # either form, whichever measured faster
    tuned = lin(x)
    lin.fused[8] = dict(cluster_splits=4, small_smem=True)
    assert lin.kernels(8) == 1
    fused = lin(x)
    lin.fused[8] = {}
    lin.cfg[8] = dict(cluster_splits=4, small_smem=True)
    assert lin.kernels(8) == 2
    two = lin(x)
    torch.cuda.synchronize()
    assert torch.equal(fused, two)  # same schedule: same bits with or without the epilogue
    assert rel_err(tuned, fused) <= 2 ** -7
