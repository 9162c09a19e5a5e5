"""Plain-PyTorch fp32 statements of every op, used as numerical oracles by the tests and benches.

The fused-op oracle is the reference's check: fp32 sum of the 16-bit inputs (NCCL all-reduce in
fp32 on GPU, gloo on CPU), residual add and RMSNorm in fp32 (exp/M17_epoch_ab/bench_ab.py:137-164),
relative error ``max|out - ref| / max|ref| <= 2^-5``.
"""
from __future__ import annotations

import torch

TOL = 2.0 ** -5


def rel_err(a: torch.Tensor, ref: torch.Tensor) -> float:
    a, ref = a.float(), ref.float()
    den = ref.abs().max().clamp_min(1e-30)
    return float((a - ref).abs().max() / den)


def rmsnorm_ref(x: torch.Tensor, gamma: torch.Tensor, eps: float) -> torch.Tensor:
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()


def fused_allreduce_add_rmsnorm_ref(xs, residual: torch.Tensor, gamma: torch.Tensor, eps: float):
    """xs: sequence (or leading dim) of per-rank partial sums. Returns fp32 (out, new_residual)."""
    total = sum(x.float() for x in xs)
    h = residual.float() + total
    return rmsnorm_ref(h, gamma, eps), h


def dist_fused_allreduce_add_rmsnorm_ref(x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor, eps: float,
                                         group=None):
    """Distributed oracle (works on gloo and NCCL): fp32 all-reduce, then add + RMSNorm in fp32."""
    import torch.distributed as dist

    total = x.float().clone()
    dist.all_reduce(total, group=group)
    h = residual.float() + total
    return rmsnorm_ref(h, gamma, eps), h


def rope_tables(max_pos: int, head_dim: int, theta: float, device=None):
    """cos/sin tables [max_pos, head_dim/2] fp32 for rotate-half RoPE."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return ang.cos().float().to(device), ang.sin().float().to(device)


def rope_ref(x: torch.Tensor, positions: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, heads, D] rotated by position (rotate-half convention)."""
    x = x.float()
    half = x.shape[-1] // 2
    c = cos[positions.long()][:, None, :]
    s = sin[positions.long()][:, None, :]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def silu_mul_ref(gu: torch.Tensor) -> torch.Tensor:
    g, u = gu.float().chunk(2, dim=-1)
    return torch.nn.functional.silu(g) * u


def paged_attention_ref(q, k_cache, v_cache, block_tables, seq_lens, scale):
    """q [B, nq, D]; caches [blocks, nkv, bs, D]; returns fp32 [B, nq, D]."""
    B, nq, D = q.shape
    nkv, bs = k_cache.shape[1], k_cache.shape[2]
    G = nq // nkv
    out = torch.empty(B, nq, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        L = int(seq_lens[b])
        nb = (L + bs - 1) // bs
        blocks = block_tables[b, :nb].long()
        k = k_cache[blocks].float().permute(1, 0, 2, 3).reshape(nkv, nb * bs, D)[:, :L]
        v = v_cache[blocks].float().permute(1, 0, 2, 3).reshape(nkv, nb * bs, D)[:, :L]
        qq = q[b].float().view(nkv, G, D)
        s = torch.einsum("hgd,htd->hgt", qq, k) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("hgt,htd->hgd", p, v).reshape(nq, D)
    return out
