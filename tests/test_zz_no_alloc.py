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


def _lib():
    native()  # loads the extension (and the torch libraries it links against)
    so = glob.glob(str(Path(K.__file__).resolve().parents[1] / "_C*.so"))
    assert so, "native extension not built"
    lib = ctypes.CDLL(so[0])
    fn = lib.cob_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 8 + [ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    lib.cob_noalloc_scratch_capacity.restype = ctypes.c_size_t
    lib.cob_noalloc_last_error.restype = ctypes.c_char_p
    return lib


def _inputs(dev, B, nq, nkv, seed):
    D, bs, maxb = 128, 16, 40
    g = torch.Generator(device=dev).manual_seed(seed)
    kc = torch.randn(B * maxb, nkv, bs, D, device=dev, generator=g).to(torch.bfloat16)
    vc = torch.randn(B * maxb, nkv, bs, D, device=dev, generator=g).to(torch.bfloat16)
    bt = torch.randperm(B * maxb, device=dev).to(torch.int32).view(B, maxb)
    seq = torch.randint(1, maxb * bs, (B,), device=dev, generator=g).to(torch.int32)
    q = torch.randn(B, nq, D, device=dev, generator=g).to(torch.bfloat16)
    return q, kc, vc, bt, seq


def _call(lib, q, kc, vc, bt, seq, out, splits, pps, scale):
    B, nq, D = q.shape
    return lib.cob_decode_attention_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), seq.data_ptr(), out.data_ptr(), B, nq,
        kc.shape[1], D, kc.shape[2], bt.shape[1], splits, pps, scale, 2, torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_regular_entry_two_calls(cuda):
    lib = _lib()
    assert lib.cob_noalloc_scratch_capacity() == 8 << 20
    scale = 1 / math.sqrt(128)
    for seed in (11, 12):  # two calls in a row share the scratch array
        q, kc, vc, bt, seq = _inputs(cuda, 6, 8, 1, seed)
        attn = K.DecodeAttention(6, 8, 1, 128, bt.shape[1], cuda)
        expect = torch.empty_like(q)
        attn(q, kc, vc, bt, seq, expect, scale)
        got = torch.full_like(q, float("nan"))
        rc = _call(lib, q, kc, vc, bt, seq, got, attn.splits, attn.pps, scale)
        torch.cuda.synchronize()
        assert rc == 0, lib.cob_noalloc_last_error()
        assert rel_err(got, expect) <= 2 ** -7
        assert rel_err(got, paged_attention_ref(q, kc, vc, bt, seq, scale)) <= 2 ** -7


def test_noalloc_rejects_oversized_geometry(cuda):
    lib = _lib()
    q, kc, vc, bt, seq = _inputs(cuda, 2, 8, 1, 3)
    out = torch.empty_like(q)
    # 2 sequences x 1 head x 4096 splits x 8 heads x 128 x 4 bytes = 32 MiB > 8 MiB
    rc = _call(lib, q, kc, vc, bt, seq, out, 4096, 1, 0.1)
    assert rc != 0
    assert b"exceeds the built-in limit" in lib.cob_noalloc_last_error()
