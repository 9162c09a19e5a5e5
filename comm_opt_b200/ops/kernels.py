"""Python wrappers of the native single-GPU decode kernels (comm_opt_b200._C)."""
from __future__ import annotations

import torch

from .._ext import native


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty_like(x) if out is None else out
    native().rmsnorm(x, gamma, out, float(eps))
    return out


def add_rmsnorm(x, residual, gamma, eps, out=None):
    """residual += x (in place); returns RMSNorm(residual) * gamma."""
    out = torch.empty_like(x) if out is None else out
    native().add_rmsnorm(x, residual, gamma, out, float(eps))
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device) if out is None else out
    native().embedding(ids, table, out)
    return out


def rope_append_kv(qkv, positions, cos, sin, block_tables, q_out, k_cache, v_cache, nq: int, nkv: int):
    native().rope_append_kv(qkv, positions, cos, sin, block_tables, q_out, k_cache, v_cache, nq, nkv)
    return q_out


def silu_mul(gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    inter = gu.shape[-1] // 2
    out = torch.empty(gu.shape[0], inter, dtype=gu.dtype, device=gu.device) if out is None else out
    native().silu_mul(gu, out)
    return out


def argmax_local(logits: torch.Tensor, vocab_offset: int, words: torch.Tensor | None = None) -> torch.Tensor:
    words = torch.empty(logits.shape[0], 2, dtype=torch.int32, device=logits.device) if words is None else words
    native().argmax_local(logits, words, int(vocab_offset))
    return words


def argmax_combine(words: torch.Tensor, world: int, ids: torch.Tensor | None = None, positions=None,
                   seq_lens=None) -> torch.Tensor:
    """Global greedy token per row from every rank's (max, index) words; optionally advances the
    decode positions / sequence lengths in the same kernel."""
    rows = words.shape[-2]
    ids = torch.empty(rows, dtype=torch.int32, device=words.device) if ids is None else ids
    native().argmax_combine(words, ids, int(world), positions, seq_lens)
    return ids


def attention_split_plan(batch: int, nkv: int, max_pages: int, num_sms: int = 148) -> tuple[int, int]:
    """Split-KV geometry: about two CTAs per SM over (batch, kv head, split)."""
    pairs = max(1, batch * nkv)
    splits = max(1, min(max_pages, (2 * num_sms + pairs - 1) // pairs))
    pps = (max_pages + splits - 1) // splits
    splits = (max_pages + pps - 1) // pps
    return splits, pps


class DecodeAttention:
    """Paged GQA decode attention with its own split-KV scratch (allocated once, graph-safe)."""

    def __init__(self, batch: int, nq: int, nkv: int, head_dim: int, max_pages: int, device, num_sms: int = 148):
        self.splits, self.pps = attention_split_plan(batch, nkv, max_pages, num_sms)
        self.batch, self.nq, self.nkv, self.head_dim = batch, nq, nkv, head_dim
        nbytes = native().attn_scratch_bytes(batch, nkv, self.splits, nq // nkv, head_dim)
        self.scratch = torch.zeros(nbytes, dtype=torch.uint8, device=device)

    def __call__(self, q, k_cache, v_cache, block_tables, seq_lens, out, scale: float):
        native().decode_attention(q, k_cache, v_cache, block_tables, seq_lens, out, self.scratch, self.splits,
                                  self.pps, float(scale))
        return out
