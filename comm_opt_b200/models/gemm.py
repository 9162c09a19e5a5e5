"""Projection layers of the decode runner.

``Linear(weight, impl="cob")`` runs the sm_100a tcgen05 swap-AB GEMM (csrc/gemm_sm100.cu);
``impl="torch"`` is the cuBLAS baseline used only for comparisons.
"""
from __future__ import annotations

import torch

from .._ext import native

_STATE: dict[int, dict] = {}
MAX_TILES = 1 << 14


def _state(device) -> dict:
    """Per-device GEMM scratch: error word, stream-K partial-tile workspace (sized for the widest
    batch tile on every SM), per-tile arrival counters (zero between calls; the kernel restores them)."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _STATE:
        sms = torch.cuda.get_device_properties(idx).multi_processor_count
        _STATE[idx] = dict(
            err=torch.zeros(1, dtype=torch.int32, device=dev),
            ws=torch.empty(sms * 2 * 128 * 256, dtype=torch.float32, device=dev),
            ctr=torch.zeros(MAX_TILES, dtype=torch.int32, device=dev),
        )
    return _STATE[idx]


def gemm_error_word(device) -> torch.Tensor:
    """Per-device int32 that a GEMM sets when one of its bounded waits times out."""
    return _state(device)["err"]


def gemm(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, ctas: int = 0, pdl: bool = False,
         small_smem: bool = False, timeout_ms: float = 2000.0) -> torch.Tensor:
    """out[M, N] = x[M, K] @ w[N, K]^T (bf16/fp16, fp32 accumulation); M <= 256 per launch."""
    M, N = x.shape[0], w.shape[0]
    out = torch.empty(M, N, dtype=x.dtype, device=x.device) if out is None else out
    st = _state(x.device)
    for m0 in range(0, M, 256):
        m1 = min(M, m0 + 256)
        native().gemm(x[m0:m1], w, out[m0:m1], st["ws"], st["ctr"], st["err"], ctas, pdl, small_smem,
                      int(timeout_ms * 1e6))
    return out


class Linear:
    def __init__(self, weight: torch.Tensor, impl: str = "cob", pdl: bool = False):
        assert impl in ("cob", "torch")
        self.weight, self.impl, self.pdl = weight, impl, pdl

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if self.impl == "torch":
            if out is None:
                return x @ self.weight.t()
            return torch.matmul(x, self.weight.t(), out=out)
        return gemm(x, self.weight, out, pdl=self.pdl)
