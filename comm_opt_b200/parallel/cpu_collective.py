"""CPU (gloo) statement of the two-shot fused algorithm of csrc/fused_ar.cu.

Same decomposition as the kernel: rank r owns columns [r*S, (r+1)*S) of every row; it sums every
rank's slice (fixed rank order) plus the residual slice, rounds h to the working dtype, computes
the partial sum of squares of its slice, then every rank gathers all h slices and all partials
and normalises locally. Checks on CPU that the column-sharded partial-sum form equals the
row-wise RMSNorm of the full sum (the reference shards rows instead, fused_ar_norm_nf.cu:103-104).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def twoshot_fused_cpu(x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor, eps: float, group=None):
    W = dist.get_world_size(group)
    r = dist.get_rank(group)
    H = x.shape[-1]
    assert H % W == 0
    S = H // W
    xs = x.float()
    # reduce-scatter by column slices: all_gather then pick the owned slice of each rank
    full = [torch.empty_like(xs) for _ in range(W)]
    dist.all_gather(full, xs.contiguous(), group=group)
    acc = torch.zeros_like(xs[..., :S])
    for src in range(W):  # fixed order, identical on every rank
        acc += full[src][..., r * S:(r + 1) * S]
    h = (acc + residual[..., r * S:(r + 1) * S].float()).to(x.dtype)
    partial = h.float().pow(2).sum(-1)
    hs = [torch.empty_like(h) for _ in range(W)]
    ps = [torch.empty_like(partial) for _ in range(W)]
    dist.all_gather(hs, h.contiguous(), group=group)
    dist.all_gather(ps, partial.contiguous(), group=group)
    hf = torch.cat(hs, dim=-1).float()
    tot = torch.zeros_like(partial)
    for p in ps:
        tot += p
    rstd = torch.rsqrt(tot / H + eps)
    out = (hf * rstd[..., None] * gamma.float()).to(x.dtype)
    return out, hf.to(x.dtype)


def layer_boundary_cpu(x: torch.Tensor, w_row: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor,
                       w_col: torch.Tensor, eps: float, pieces: int = 3, splits: int = 2, group=None):
    """CPU statement of the layer-boundary kernels of csrc/fused_gemm.cu (gemm_push -> ar_norm_gemm).

    x [M, K1] and w_row [H, K1] are this rank's row-parallel shard; w_col [N, H] its column-parallel
    shard. Push: y_r = bf16(x w_row^T) lands on every rank. Consumer: the H columns are cut into
    `splits` K-ranges of `pieces` pieces each; a piece sums the landed partials of its columns in rank
    order plus the residual (h rounded to the working dtype), keeps a per-row sum of squares; the
    GEMM runs on bf16(h * gamma) split by split, and the output is scaled per row by
    rsqrt(sum of all pieces' sums / H + eps) - RMSNorm folded into the GEMM. Returns (z, h)."""
    W = dist.get_world_size(group)
    y = (x.float() @ w_row.float().t()).to(x.dtype)
    ys = [torch.empty_like(y) for _ in range(W)]
    dist.all_gather(ys, y.contiguous(), group=group)
    H = y.shape[-1]
    h = torch.empty_like(residual)
    a = torch.empty(residual.shape, dtype=x.dtype)
    ss = []
    for r in range(splits):
        c0, c1 = r * H // splits, (r + 1) * H // splits
        for t in range(pieces):
            lo, hi = c0 + (c1 - c0) * t // pieces, c0 + (c1 - c0) * (t + 1) // pieces
            acc = residual[..., lo:hi].float().clone()
            for src in range(W):  # fixed order, identical on every rank
                acc += ys[src][..., lo:hi].float()
            hp = acc.to(x.dtype)
            h[..., lo:hi] = hp
            ss.append(hp.float().pow(2).sum(-1))
            a[..., lo:hi] = (hp.float() * gamma[lo:hi].float()).to(x.dtype)
    rstd = torch.rsqrt(sum(ss) / H + eps)
    z = torch.zeros(residual.shape[:-1] + (w_col.shape[0],))
    for r in range(splits):  # split-K partial GEMMs, summed in split order
        c0, c1 = r * H // splits, (r + 1) * H // splits
        z += a[..., c0:c1].float() @ w_col[:, c0:c1].float().t()
    return (z * rstd[..., None]).to(x.dtype), h
