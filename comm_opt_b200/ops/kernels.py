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


def rope_append_kv(qkv, positions, cos, sin, block_tables, q_out, k_cache, v_cache, nq: int, nkv: int, bias=None):
    """RoPE on q and k of the fused qkv rows, q to q_out, k and v into the paged caches; `bias`
    ([(nq + 2 nkv) * head_dim], optional) is the QKV projection's bias, added first."""
    native().rope_append_kv(qkv, positions, cos, sin, block_tables, q_out, k_cache, v_cache, nq, nkv, bias)
    return q_out


def silu_mul(gu: torch.Tensor, out: torch.Tensor | None = None, interleave: int = 0) -> torch.Tensor:
    """out[M, I] = silu(gate) * up of gu [M, 2I]: [gate | up] halves, or with `interleave` = c blocks of c
    gate then c up features (the layout of gate/up weights packed with `pack_weight(w, interleave=c)`)."""
    inter = gu.shape[-1] // 2
    out = torch.empty(gu.shape[0], inter, dtype=gu.dtype, device=gu.device) if out is None else out
    native().silu_mul(gu, out, int(interleave))
    return out


def set_l2_prefetch(tiles: int) -> int:
    """Weight tiles beyond its shared-memory ring that every GEMM of this package prefetches into L2
    before it waits for its activations (0 = none); returns the old value. Read at launch time, so a
    CUDA graph keeps the value it was captured with."""
    old = native().get_l2_prefetch()
    native().set_l2_prefetch(int(tiles))
    return old


def set_attn_stages(n: int) -> int:
    """KV pages in flight per warp of the decode attention kernel: 6 (the deep ring, one CTA per SM; used
    where the grid fits one wave at one CTA per SM) or 3 (two CTAs per SM). Read at launch time (a CUDA
    graph keeps the launch it captured); returns the old setting."""
    return int(native().set_attn_stages(int(n)))


def set_pdl(on: bool) -> bool:
    """Launch every kernel of this package with programmatic dependent launch (returns the old value)."""
    old = native().get_pdl()
    native().set_pdl(bool(on))
    return old


def argmax_local(logits: torch.Tensor, vocab_offset: int, keys: torch.Tensor | None = None) -> torch.Tensor:
    """Fold the row maxima of this rank's vocabulary shard into int64 keys (zero before use)."""
    keys = torch.zeros(logits.shape[0], dtype=torch.int64, device=logits.device) if keys is None else keys
    native().argmax_local(logits, keys, int(vocab_offset))
    return keys


def argmax_combine(gathered: torch.Tensor, world: int, ids: torch.Tensor | None = None, positions=None,
                   seq_lens=None, local_keys=None) -> torch.Tensor:
    """Global greedy token per row from every rank's keys [world, rows]; optionally advances the decode
    positions / sequence lengths and clears this rank's keys in the same kernel."""
    rows = gathered.shape[-1]
    ids = torch.empty(rows, dtype=torch.int32, device=gathered.device) if ids is None else ids
    native().argmax_combine(gathered, ids, int(world), positions, seq_lens, local_keys)
    return ids


ATTN_CTAS_PER_SM = 2  # the kernel's shared memory (104-114 KB with the push merge) allows two CTAs per SM


def attention_split_plan(batch: int, nkv: int, max_pages: int, num_sms: int = 148) -> tuple[int, int, bool]:
    """Split-KV geometry (splits, pages per split, cluster merge).

    As many CTAs over (batch, kv head, split) as fit in ONE wave of resident CTAs (a partial second
    wave would double the kernel time), but merged inside a thread-block cluster (distributed shared
    memory) wherever possible: when one wave allows more than 8 splits per pair, 8 splits while each
    CTA keeps at most 32 pages, else 16 (a non-portable cluster size the kernel supports) if 16 still
    fit one wave. Only sequences longer than 16 x 512 pages use more splits and the global merge."""
    pairs = max(1, batch * nkv)
    slots = ATTN_CTAS_PER_SM * num_sms
    splits = max(1, min(max_pages, slots // pairs))
    if splits > 8:
        # Measured at batch 8, one KV head (CUDA graphs, one B200): 2048 tokens - 8 splits 9.9 us, 16
        # 10.8 us, 32 with the global merge 26.4 us; 8192 tokens - 8 splits 18.6 us, 37 with the global
        # merge 34.4 us (the global merge, one CTA folding every split, costs more than a longer chain)
        splits = 16 if (max_pages + 7) // 8 > 32 and pairs * 16 <= slots else 8
    pps = min(512, (max_pages + splits - 1) // splits)
    splits = (max_pages + pps - 1) // pps
    return splits, pps, 1 < splits <= 16


class DecodeAttention:
    """Paged GQA decode attention with its own split-KV scratch (allocated once, graph-safe)."""

    def __init__(self, batch: int, nq: int, nkv: int, head_dim: int, max_pages: int, device, num_sms: int = 148):
        self.splits, self.pps, self.cluster = attention_split_plan(batch, nkv, max_pages, num_sms)
        self.batch, self.nq, self.nkv, self.head_dim = batch, nq, nkv, head_dim
        nbytes = native().attn_scratch_bytes(batch, nkv, self.splits, nq // nkv, head_dim)
        self.scratch = torch.zeros(nbytes, dtype=torch.uint8, device=device)

    def __call__(self, q, k_cache, v_cache, block_tables, seq_lens, out, scale: float, append: dict | None = None):
        """`append` (keys qkv, positions, cos, sin, optional bias): RoPE + KV append of the new token in the
        same kernel - the query and the new k / v head come from the QKV projection output `qkv`
        [B, (nq + 2 nkv) * D], the new k / v are written into the caches at `positions` (`q` is not read)."""
        a = append or {}
        native().decode_attention(q, k_cache, v_cache, block_tables, seq_lens, out, self.scratch, self.splits,
                                  self.pps, float(scale), self.cluster, qkv=a.get("qkv"), qkv_bias=a.get("bias"),
                                  positions=a.get("positions"), cos=a.get("cos"), sin=a.get("sin"))
        return out
