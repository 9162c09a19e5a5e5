"""Allocation-free attention entry point, called through its exported C symbol.

The entry point serves callers that cannot allocate device memory while they decode (C or other
language runtimes without PyTorch's caching allocator, where cudaMalloc would synchronize the
device; serving engines that reserve all device memory for weights and KV cache up front). Its
split-KV scratch is a fixed array inside the library. This file is collected last on purpose, and
it must pass both alone in a fresh process and after every other test.
"""
import ctypes
import glob
import math
from pathlib import Path

import pytest
import torch

import comm_opt_b200.ops.kernels as K
from comm_opt_b200._ext import native
from comm_opt_b200.ops.reference import paged_attention_ref, rel_err

pytestmark = pytest.mark.gpu

DT = {torch.float16: 1, torch.bfloat16: 2}


def _lib():
    native()  # loads the extension (and the torch libraries it links against)
    so = glob.glob(str(Path(K.__file__).resolve().parents[1] / "_C*.so"))
    assert so, "native extension not built"
    lib = ctypes.CDLL(so[0])
    fn = lib.cob_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 9 + [ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    lib.cob_noalloc_scratch_capacity.restype = ctypes.c_size_t
    lib.cob_noalloc_last_error.restype = ctypes.c_char_p
    return lib


def _inputs(dev, B, nq, nkv, seed, D=128, dtype=torch.bfloat16, maxb=40):
    bs = 16
    g = torch.Generator(device=dev).manual_seed(seed)
    kc = torch.randn(B * maxb, nkv, bs, D, device=dev, generator=g).to(dtype)
    vc = torch.randn(B * maxb, nkv, bs, D, device=dev, generator=g).to(dtype)
    bt = torch.randperm(B * maxb, device=dev).to(torch.int32).view(B, maxb)
    seq = torch.randint(1, maxb * bs, (B,), device=dev, generator=g).to(torch.int32)
    q = torch.randn(B, nq, D, device=dev, generator=g).to(dtype)
    return q, kc, vc, bt, seq


def _call(lib, q, kc, vc, bt, seq, out, splits, pps, scale, **override):
    B, nq, D = q.shape
    a = dict(batch=B, nq=nq, nkv=kc.shape[1], head_dim=D, block_size=kc.shape[2], max_blocks=bt.shape[1],
             num_blocks=kc.shape[0], splits=splits, pps=pps)
    a.update(override)
    return lib.cob_decode_attention_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), seq.data_ptr(), out.data_ptr(), a["batch"],
        a["nq"], a["nkv"], a["head_dim"], a["block_size"], a["max_blocks"], a["num_blocks"], a["splits"], a["pps"],
        scale, DT[q.dtype], torch.cuda.current_stream().cuda_stream)


def _check_against_regular(lib, dev, B, nq, nkv, seed, D=128, dtype=torch.bfloat16, splits=None):
    q, kc, vc, bt, seq = _inputs(dev, B, nq, nkv, seed, D, dtype)
    scale = 1 / math.sqrt(D)
    attn = K.DecodeAttention(B, nq, nkv, D, bt.shape[1], dev)
    expect = torch.empty_like(q)
    attn(q, kc, vc, bt, seq, expect, scale)
    if splits is None:
        splits, pps = attn.splits, attn.pps
    else:
        pps = (bt.shape[1] + splits - 1) // splits
    got = torch.full_like(q, float("nan"))
    rc = _call(lib, q, kc, vc, bt, seq, got, splits, pps, scale)
    torch.cuda.synchronize()
    assert rc == 0, lib.cob_noalloc_last_error()
    tol = 2 ** -7  # the attention tests' tolerance for 16-bit outputs
    assert rel_err(got, expect) <= tol
    assert rel_err(got, paged_attention_ref(q, kc, vc, bt, seq, scale)) <= tol
    return splits


def test_noalloc_matches_regular_entry_two_calls(cuda):
    """Two calls in a row on the shared array; the second has a different batch, head count and split
    count, so its arrival counters sit where the first call left partial outputs (they must be
    cleared by the call, not assumed zero)."""
    lib = _lib()
    assert lib.cob_noalloc_scratch_capacity() == 8 << 20
    s1 = _check_against_regular(lib, cuda, 6, 8, 1, 11, splits=20)
    s2 = _check_against_regular(lib, cuda, 3, 16, 2, 12, splits=5)
    assert (6 * 1 * s1) > (3 * 2 * s2)  # second call's counters land inside the first call's partials


def test_noalloc_fp16_head_dim_64_many_kv_heads(cuda):
    lib = _lib()
    _check_against_regular(lib, cuda, 2, 16, 4, 21, D=64, dtype=torch.float16)
    _check_against_regular(lib, cuda, 4, 8, 2, 22, D=128, dtype=torch.float16)


def test_noalloc_rejects_bad_arguments(cuda):
    lib = _lib()
    q, kc, vc, bt, seq = _inputs(cuda, 2, 8, 1, 3)
    out = torch.empty_like(q)
    # 2 sequences x 1 head x 4096 splits x 8 heads x 128 x 4 bytes = 32 MiB > 8 MiB
    assert _call(lib, q, kc, vc, bt, seq, out, 4096, 1, 0.1) != 0
    assert b"exceeds the built-in limit" in lib.cob_noalloc_last_error()
    # 4 splits x 8 pages cover 32 of the 40 block-table columns: tokens would be dropped
    assert _call(lib, q, kc, vc, bt, seq, out, 4, 8, 0.1) != 0
    assert b"does not cover max_blocks_per_seq" in lib.cob_noalloc_last_error()
    assert _call(lib, q, kc, vc, bt, seq, out, 4, 10, 0.1, num_blocks=0) != 0
    assert b"num_blocks" in lib.cob_noalloc_last_error()
    assert _call(lib, q, kc, vc, bt, seq, out, 4, 10, 0.1, block_size=32) != 0
    assert b"block_size must be 16" in lib.cob_noalloc_last_error()
    assert _call(lib, q, kc, vc, bt, seq, out, 4, 10, 0.1, head_dim=96) != 0
    assert b"head_dim" in lib.cob_noalloc_last_error()
    torch.cuda.synchronize()  # nothing was launched by the rejected calls
