"""Functional API with the reference's call semantics (exp/M17_epoch_ab/fused_ar_norm_nf.cu:203-206):

    out, new_residual = fused_allreduce_add_rmsnorm(x, residual, gamma, eps)

x is this rank's partial sum [T, H], residual [T, H] is replicated (updated in place and returned),
out = RMSNorm(residual + sum_ranks(x)) * gamma. On CUDA tensors the call runs this package's fused kernel
through a communicator kept per (process group, device, dtype) and grown (collectively: every rank of a
TP group calls with the same shapes) when a call exceeds its capacity. On CPU tensors it runs the
column-sharded two-shot statement over the group's gloo backend (or the single-rank formula), so the
same code runs in CPU tests.

    layer_boundary(x, w_row, residual, gamma, w_col, eps)  ->  (z, new_residual)

is the fused row-parallel GEMM -> all-reduce + residual + RMSNorm -> column-parallel GEMM of one layer
boundary (two kernels on CUDA; the same math stated with torch.distributed on CPU).
"""
from __future__ import annotations

import torch

from .parallel.communicator import TPCommunicator
from .parallel.config import CommConfig

_COMMS: dict[tuple, TPCommunicator] = {}


def _group_key(group):
    import torch.distributed as dist

    if group is None and dist.is_available() and dist.is_initialized():
        group = dist.group.WORLD
    return group, (id(group) if group is not None else None)


def _world(group) -> int:
    import torch.distributed as dist

    return dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1


def communicator(x: torch.Tensor, hidden: int, rows: int, group=None, config: CommConfig | None = None,
                 factory=TPCommunicator.from_config) -> TPCommunicator:
    """The cached communicator for (group, device, dtype), rebuilt with doubled capacity when needed."""
    group, gid = _group_key(group)
    key = (gid, x.device, x.dtype)
    comm = _COMMS.get(key)
    if comm is not None and (rows > comm.max_rows or hidden > comm.max_hidden):
        cfg = CommConfig.from_dict(dict(config.kwargs() if config else CommConfig.from_env().kwargs(),
                                        max_rows=max(rows, 2 * comm.max_rows),
                                        max_hidden=max(hidden, comm.max_hidden)))
        comm.close()
        comm = None
        config = cfg
    if comm is None:
        cfg = config or CommConfig.from_env()
        if rows > cfg.max_rows or hidden > cfg.max_hidden:
            cfg = CommConfig.from_dict(dict(cfg.kwargs(), max_rows=max(rows, cfg.max_rows),
                                            max_hidden=max(hidden, cfg.max_hidden)))
        comm = factory(group, cfg, device=x.device, dtype=x.dtype)
        _COMMS[key] = comm
    return comm


def fused_allreduce_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-6,
                                group=None, config: CommConfig | None = None, variant="auto"):
    """Returns (out, new_residual); `residual` is updated in place."""
    if not x.is_cuda:
        from .parallel.cpu_collective import twoshot_fused_cpu

        if _world(group) == 1:
            h = (x.float() + residual.float()).to(x.dtype)
            out = (h.float() * torch.rsqrt(h.float().pow(2).mean(-1, keepdim=True) + eps) * gamma.float()).to(x.dtype)
        else:
            out, h = twoshot_fused_cpu(x, residual, gamma, eps, group=_group_key(group)[0])
        residual.copy_(h)
        return out, residual
    rows = x.numel() // x.shape[-1]
    comm = communicator(x, x.shape[-1], rows, group, config)
    return comm.fused_allreduce_add_rmsnorm(x, residual, gamma, eps, variant=variant)


def layer_boundary(x: torch.Tensor, w_row: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor,
                   w_col: torch.Tensor, eps: float = 1e-6, group=None, config: CommConfig | None = None):
    """Row-parallel GEMM (x [M, K1] @ w_row[H, K1]^T) -> all-reduce + residual + RMSNorm -> column-parallel
    GEMM (@ w_col[N, H]^T). Returns (z [M, N], new_residual); `residual` is updated in place."""
    if not x.is_cuda:
        import torch.distributed as dist

        y = x.float() @ w_row.float().t()
        if _world(group) > 1:
            dist.all_reduce(y, group=_group_key(group)[0])
        h = (residual.float() + y).to(residual.dtype)
        n = h.float() * torch.rsqrt(h.float().pow(2).mean(-1, keepdim=True) + eps) * gamma.float()
        residual.copy_(h)
        return (n @ w_col.float().t()).to(x.dtype), residual
    comm = communicator(residual, residual.shape[-1], residual.numel() // residual.shape[-1], group, config)
    if comm.world == 1:
        y = torch.matmul(x, w_row.t())
        h = residual.float() + y.float()
        residual.copy_(h.to(residual.dtype))
        n = (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps) * gamma.float()).to(x.dtype)
        return torch.matmul(n, w_col.t()), residual
    comm.prepare_fused_gemm(residual.shape[-1])
    comm.gemm_push(x, w_row)
    return comm.ar_norm_gemm(residual, gamma, w_col, eps), residual


def release():
    """Close every cached communicator (collective: call on every rank)."""
    for comm in _COMMS.values():
        comm.close()
    _COMMS.clear()
