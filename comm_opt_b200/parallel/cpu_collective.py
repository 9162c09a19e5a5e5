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
