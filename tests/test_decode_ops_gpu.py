"""Numerics of the single-GPU decode kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch

from comm_opt_b200.ops import kernels as K
from comm_opt_b200.ops.reference import paged_attention_ref, rel_err, rmsnorm_ref, rope_ref, rope_tables, silu_mul_ref

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float16, torch.float32]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,hidden", [(1, 8192), (7, 4096), (64, 5120), (3, 16384)])
def test_rmsnorm_and_add(cuda, dtype, rows, hidden):
    x = torch.randn(rows, hidden, device=cuda).to(dtype)
    r0 = torch.randn(rows, hidden, device=cuda).to(dtype)
    g = (1 + 0.1 * torch.randn(hidden, device=cuda)).to(dtype)
    tol = 1e-5 if dtype == torch.float32 else 2 ** -7
    assert rel_err(K.rmsnorm(x, g, 1e-5), rmsnorm_ref(x, g, 1e-5)) <= tol
    res = r0.clone()
    out = K.add_rmsnorm(x, res, g, 1e-5)
    h = (x.float() + r0.float())
    assert rel_err(res, h) <= tol
    assert rel_err(out, rmsnorm_ref(res.float(), g, 1e-5)) <= tol


def test_embedding(cuda):
    table = torch.randn(1000, 4096, device=cuda).to(torch.bfloat16)
    ids = torch.tensor([0, 999, 5, 5, 123], device=cuda, dtype=torch.int32)
    assert torch.equal(K.embedding(ids, table), table[ids.long()])


@pytest.mark.parametrize("nq,nkv,bias", [(8, 1, False), (32, 8, False), (4, 4, False), (5, 1, True), (20, 4, True)])
def test_rope_append_kv(cuda, nq, nkv, bias):
    """RoPE + paged append against fp32; with `bias` (the Qwen2.5 QKV bias, 5 query heads per KV head at
    TP=8 / TP=2) added to q, k and v before the rotation."""
    B, D, bs, maxb = 5, 128, 16, 8
    dtype = torch.bfloat16
    cos, sin = rope_tables(maxb * bs, D, 500000.0, cuda)
    qkv = torch.randn(B, (nq + 2 * nkv) * D, device=cuda).to(dtype)
    b_qkv = torch.randn((nq + 2 * nkv) * D, device=cuda).to(dtype) if bias else None
    pos = torch.tensor([0, 17, 33, 127, 64], device=cuda, dtype=torch.int32)
    bt = torch.randperm(B * maxb, device=cuda).to(torch.int32).view(B, maxb)
    kc = torch.zeros(B * maxb, nkv, bs, D, device=cuda, dtype=dtype)
    vc = torch.zeros_like(kc)
    q = torch.empty(B, nq, D, device=cuda, dtype=dtype)
    K.rope_append_kv(qkv, pos, cos, sin, bt, q, kc, vc, nq, nkv, bias=b_qkv)
    heads = (qkv.float() + (b_qkv.float() if bias else 0.0)).view(B, nq + 2 * nkv, D)
    assert rel_err(q, rope_ref(heads[:, :nq], pos, cos, sin)) <= 2 ** -7
    kref = rope_ref(heads[:, nq:nq + nkv], pos, cos, sin)
    for b in range(B):
        p = int(pos[b])
        blk = int(bt[b, p // bs])
        assert rel_err(kc[blk, :, p % bs], kref[b]) <= 2 ** -7
        if bias:
            assert rel_err(vc[blk, :, p % bs], heads[b, nq + nkv:]) <= 2 ** -7
        else:
            assert torch.equal(vc[blk, :, p % bs], heads[b, nq + nkv:].to(dtype))


@pytest.mark.parametrize("dtype", DTYPES)
def test_silu_mul(cuda, dtype):
    gu = torch.randn(9, 2 * 3584, device=cuda).to(dtype)
    tol = 1e-5 if dtype == torch.float32 else 2 ** -7
    assert rel_err(K.silu_mul(gu), silu_mul_ref(gu)) <= tol


@pytest.mark.parametrize("dtype", DTYPES)
def test_silu_mul_interleaved(cuda, dtype):
    """Gate/up rows interleaved in blocks of 64 (the packed gate/up weights' output order)."""
    from comm_opt_b200.models.gemm import interleave_rows

    gu = torch.randn(5, 2 * 3584, device=cuda).to(dtype)
    il = interleave_rows(gu.t().contiguous(), 64).t().contiguous()  # columns in the interleaved order
    assert torch.equal(K.silu_mul(il, interleave=64), K.silu_mul(gu))


def test_argmax_local_and_combine(cuda):
    V, world, rows = 16032, 4, 6
    logits = torch.randn(world, rows, V, device=cuda).to(torch.bfloat16)
    logits[2, 3, 77] = 100.0  # unique max on rank 2
    keys = torch.stack([K.argmax_local(logits[r], r * V) for r in range(world)])
    local = keys[0].clone()
    ids = K.argmax_combine(keys.contiguous(), world, local_keys=local)
    ref = torch.cat(list(logits), dim=-1).float().argmax(-1)
    assert torch.equal(ids.long(), ref)
    assert int(ids[3]) == 2 * V + 77
    assert torch.all(local == 0)  # cleared for the next step
    # ties resolve to the lowest global index, negative values order correctly
    t = torch.full((2, 1, 4096), -3.0, device=cuda).to(torch.bfloat16)
    t[0, 0, 100] = -1.0
    t[1, 0, 5] = -1.0
    k2 = torch.stack([K.argmax_local(t[r], r * 4096) for r in range(2)])
    assert int(K.argmax_combine(k2.contiguous(), 2)[0]) == 100


@pytest.mark.parametrize("nq,nkv", [(8, 1), (32, 8), (16, 4)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_attention(cuda, nq, nkv, dtype):
    check_decode_attention(cuda, nq, nkv, dtype, 128)


@pytest.mark.parametrize("nq,nkv", [(4, 1), (32, 4)])
def test_decode_attention_head_dim_64(cuda, nq, nkv):
    """TinyLlama-1.1B heads (head_dim 64, 8 query heads per KV head; 4 per rank at TP=8)."""
    check_decode_attention(cuda, nq, nkv, torch.bfloat16, 64)


def check_decode_attention(cuda, nq, nkv, dtype, D):
    B, bs, maxb = 6, 16, 40
    seq = torch.tensor([1, 15, 16, 17, 300, 640], device=cuda, dtype=torch.int32)
    nblocks = B * maxb
    kc = torch.randn(nblocks, nkv, bs, D, device=cuda).to(dtype)
    vc = torch.randn(nblocks, nkv, bs, D, device=cuda).to(dtype)
    bt = torch.randperm(nblocks, device=cuda).to(torch.int32).view(B, maxb)
    q = torch.randn(B, nq, D, device=cuda).to(dtype)
    scale = 1 / math.sqrt(D)
    ref = paged_attention_ref(q, kc, vc, bt, seq, scale)
    for num_sms in (148, 8, 1):  # global split merge, cluster (DSMEM) merge, single split
        attn = K.DecodeAttention(B, nq, nkv, D, maxb, cuda, num_sms=num_sms)
        out = torch.empty_like(q)
        for _ in range(2):  # second call checks the split counters were reset
            attn(q, kc, vc, bt, seq, out, scale)
            torch.cuda.synchronize()
            assert rel_err(out, ref) <= 2 ** -7, (num_sms, attn.splits, attn.cluster, rel_err(out, ref))
    # cluster merge up to 16 splits (9..16: non-portable cluster sizes), global merge otherwise
    for splits, cl in [(2, True), (3, True), (5, True), (8, True), (10, True), (16, True), (40, False), (13, False)]:
        attn = K.DecodeAttention(B, nq, nkv, D, maxb, cuda)
        attn.splits, attn.pps, attn.cluster = splits, -(-maxb // splits), cl
        attn.splits = -(-maxb // attn.pps)
        from comm_opt_b200._ext import native

        attn.scratch = torch.zeros(native().attn_scratch_bytes(B, nkv, attn.splits, nq // nkv, D), dtype=torch.uint8,
                                   device=cuda)
        out = torch.empty_like(q)
        attn(q, kc, vc, bt, seq, out, scale)
        torch.cuda.synchronize()
        assert rel_err(out, ref) <= 2 ** -7, (splits, rel_err(out, ref))


@pytest.mark.parametrize("nq,nkv,bias,D", [(8, 1, False, 128), (32, 8, False, 128), (5, 1, True, 128),
                                           (20, 4, True, 128), (4, 1, False, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_attention_with_fused_append(cuda, nq, nkv, bias, D, dtype):
    """RoPE + KV append of the new token inside the attention kernel equals the append kernel followed by
    the attention: same output (fp32 oracle too) and the same cache rows, for the global merge, the
    cluster merge and a single split, with the new token at the start, middle and end of a page."""
    B, bs, maxb = 6, 16, 40
    seq = torch.tensor([1, 16, 17, 33, 300, 640], device=cuda, dtype=torch.int32)
    pos = seq - 1
    g = torch.Generator(device=cuda).manual_seed(nq * 3 + D)
    nblocks = B * maxb
    kc0 = torch.randn(nblocks, nkv, bs, D, device=cuda, generator=g).to(dtype)
    vc0 = torch.randn(nblocks, nkv, bs, D, device=cuda, generator=g).to(dtype)
    bt = torch.randperm(nblocks, device=cuda).to(torch.int32).view(B, maxb)
    qkv = torch.randn(B, (nq + 2 * nkv) * D, device=cuda, generator=g).to(dtype)
    b_qkv = torch.randn((nq + 2 * nkv) * D, device=cuda, generator=g).to(dtype) if bias else None
    cos, sin = rope_tables(maxb * bs, D, 500000.0, cuda)
    scale = 1 / math.sqrt(D)
    # reference path: the append kernel, then the attention
    kc1, vc1 = kc0.clone(), vc0.clone()
    q = torch.empty(B, nq, D, device=cuda, dtype=dtype)
    K.rope_append_kv(qkv, pos, cos, sin, bt, q, kc1, vc1, nq, nkv, bias=b_qkv)
    ref = paged_attention_ref(q, kc1, vc1, bt, seq, scale)
    for num_sms in (148, 8, 1):
        base = K.DecodeAttention(B, nq, nkv, D, maxb, cuda, num_sms=num_sms)
        want = torch.empty_like(q)
        base(q, kc1, vc1, bt, seq, want, scale)
        kc2, vc2 = kc0.clone(), vc0.clone()
        got = torch.full_like(q, float("nan"))
        base(torch.empty_like(q), kc2, vc2, bt, seq, got, scale,
             append=dict(qkv=qkv, positions=pos, cos=cos, sin=sin, bias=b_qkv))
        torch.cuda.synchronize()
        assert rel_err(got, want) <= 2 ** -7, (num_sms, rel_err(got, want))
        assert rel_err(got, ref) <= 2 ** -7
        assert rel_err(kc2, kc1) <= 2 ** -7 and rel_err(vc2, vc1) <= 2 ** -7


@pytest.fixture
def deep_ring():
    old = K.set_attn_stages(6)
    yield
    K.set_attn_stages(old)


@pytest.mark.parametrize("nq,nkv,D", [(8, 1, 128), (16, 4, 128), (4, 1, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_decode_attention_deep_ring(cuda, deep_ring, nq, nkv, D, dtype):
    """The deep KV ring (six pages in flight per warp, one CTA per SM) gives the shallow ring's bits: the
    same pages in the same order per warp, only requested earlier; every merge form and the fused append."""
    check_decode_attention(cuda, nq, nkv, dtype, D)
    B, bs, maxb = 6, 16, 40
    seq = torch.tensor([1, 16, 17, 33, 300, 640], device=cuda, dtype=torch.int32)
    g = torch.Generator(device=cuda).manual_seed(5)
    kc0 = torch.randn(B * maxb, nkv, bs, D, device=cuda, generator=g).to(dtype)
    vc0 = torch.randn(B * maxb, nkv, bs, D, device=cuda, generator=g).to(dtype)
    bt = torch.randperm(B * maxb, device=cuda).to(torch.int32).view(B, maxb)
    qkv = torch.randn(B, (nq + 2 * nkv) * D, device=cuda, generator=g).to(dtype)
    cos, sin = rope_tables(maxb * bs, D, 500000.0, cuda)
    app = dict(qkv=qkv, positions=seq - 1, cos=cos, sin=sin)
    for num_sms in (148, 8):  # cluster merge (deep ring), then more CTAs than that
        outs = []
        for stages in (6, 3):
            K.set_attn_stages(stages)
            attn = K.DecodeAttention(B, nq, nkv, D, maxb, cuda, num_sms=num_sms)
            kc, vc = kc0.clone(), vc0.clone()
            out = torch.empty(B, nq, D, device=cuda, dtype=dtype)
            attn(torch.empty_like(out), kc, vc, bt, seq, out, 1 / math.sqrt(D), append=app)
            torch.cuda.synchronize()
            outs.append((out, kc, vc))
        K.set_attn_stages(6)
        assert all(torch.equal(a, b) for a, b in zip(outs[0], outs[1])), num_sms
