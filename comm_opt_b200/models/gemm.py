"""Projection layers of the decode runner.

``Linear(weight, impl="cob")`` runs the sm_100a tcgen05 swap-AB GEMM (csrc/gemm_sm100.cu);
``impl="torch"`` is the cuBLAS baseline used only for comparisons.
"""
from __future__ import annotations

import torch

from .._ext import native

_STATE: dict[int, dict] = {}
MAX_TILES = 1 << 14
BM, BK = 128, 64


def _swizzle_index(device) -> torch.Tensor:
    """idx[r, c, e] = c ^ (r % 8): the 16-byte chunk of row r stored at chunk position c (128-byte swizzle)."""
    r = torch.arange(BM, device=device).view(BM, 1, 1)
    c = torch.arange(8, device=device).view(1, 8, 1)
    return (c ^ (r & 7)).expand(BM, 8, 8)


def interleave_rows(w: torch.Tensor, c: int = BM // 2) -> torch.Tensor:
    """[..., 2I, K] = [gate rows; up rows] -> blocks of c gate rows followed by the matching c up rows
    (with c = 64 every 128-row output tile of the decode GEMM holds 64 gate features and their up
    features: the layout of its SwiGLU epilogue)."""
    I2, K = w.shape[-2], w.shape[-1]
    I = I2 // 2
    if I2 % 2 or I % c:
        raise ValueError(f"gate/up rows {I2} do not split into blocks of {c}")
    lead = w.shape[:-2]
    g = w[..., :I, :].reshape(*lead, I // c, c, K)
    u = w[..., I:, :].reshape(*lead, I // c, c, K)
    return torch.stack([g, u], dim=-3).reshape(*lead, I2, K).contiguous()


def deinterleave_rows(w: torch.Tensor, c: int = BM // 2) -> torch.Tensor:
    """Inverse of `interleave_rows`."""
    I2, K = w.shape[-2], w.shape[-1]
    lead = w.shape[:-2]
    v = w.reshape(*lead, I2 // (2 * c), 2, c, K).transpose(-4, -3)
    return v.reshape(*lead, I2, K).contiguous()


class PackedWeight:
    """A weight [N, K] stored for the decode GEMMs' bulk loads: 128 x 64 blocks (16 KB for 16-bit types)
    in (output tile, k-step) order, each block laid out exactly as the 128-byte-swizzled shared-memory
    image the tensor cores read (16-byte chunk c of row r at chunk position c ^ (r % 8)); rows past N are
    zero. A CTA's share of the weight stream is then one contiguous range of memory, read by 16 KB bulk
    copies (no tensor-map descriptor, no per-row 128-byte pieces). Static weights are packed once at
    load. `ranks` > 1 stacks the weights of emulated ranks ([ranks, N, K] -> ranks x the blocks).
    `il` > 0: a gate/up weight whose rows were interleaved in blocks of `il` before packing (GEMM outputs
    come in that order; `dense()` returns the original [gate; up] rows)."""

    def __init__(self, data: torch.Tensor, n: int, k: int, ranks: int = 1, il: int = 0):
        T = (n + BM - 1) // BM
        assert data.dim() == 4 and tuple(data.shape[1:]) == (k // BK, BM, BK) and data.shape[0] == ranks * T
        self.data, self.n, self.k, self.ranks, self.il = data, n, k, ranks, il

    @property
    def shape(self) -> tuple:
        return (self.n, self.k) if self.ranks == 1 else (self.ranks, self.n, self.k)

    @property
    def dtype(self):
        return self.data.dtype

    @property
    def device(self):
        return self.data.device

    def dense(self) -> torch.Tensor:
        """The row-major weight ([N, K], or [ranks, N, K]) as a new tensor."""
        RT, KT = self.data.shape[:2]
        T = RT // self.ranks
        v = self.data.view(RT, KT, BM, 8, 8)
        idx = _swizzle_index(self.device).expand(RT, KT, BM, 8, 8)
        blocks = v.gather(3, idx)  # the same permutation undoes itself (XOR)
        w = blocks.view(self.ranks, T, KT, BM, 8, 8).permute(0, 1, 3, 2, 4, 5).reshape(self.ranks, T * BM, KT * BK)
        w = w[:, : self.n].contiguous()
        if self.il:
            w = deinterleave_rows(w, self.il)
        return w[0] if self.ranks == 1 else w


def pack_weight(w: torch.Tensor, interleave: int = 0) -> PackedWeight:
    """Pack a row-major weight [N, K] (or [ranks, N, K]), K a multiple of 64, into the decode GEMMs'
    block layout. `interleave` = c > 0: w is a [gate; up] projection whose rows are first interleaved in
    blocks of c (`interleave_rows`); c = 64 lets the GEMM's SwiGLU epilogue produce silu(gate) * up."""
    ranks = 1 if w.dim() == 2 else w.shape[0]
    if interleave:
        w = interleave_rows(w, interleave)
    w3 = w.reshape(ranks, w.shape[-2], w.shape[-1])
    _, N, K = w3.shape
    if K % BK:
        raise ValueError(f"K = {K} is not a multiple of {BK}")
    T, KT = (N + BM - 1) // BM, K // BK
    if T * BM != N:
        w3 = torch.cat([w3, w3.new_zeros(ranks, T * BM - N, K)], 1)
    v = w3.reshape(ranks * T, BM, KT, 8, 8).permute(0, 2, 1, 3, 4)
    idx = _swizzle_index(w.device).expand(ranks * T, KT, BM, 8, 8)
    return PackedWeight(v.gather(3, idx).view(ranks * T, KT, BM, BK), N, K, ranks, interleave)


def dense(w) -> torch.Tensor:
    """Row-major [N, K] form of a weight (unpacks a PackedWeight)."""
    return w.dense() if isinstance(w, PackedWeight) else w


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
         small_smem: bool = False, cluster_splits: int = 0, timeout_ms: float = 2000.0,
         swiglu: bool = False) -> torch.Tensor:
    """out[M, N] = x[M, K] @ w[N, K]^T (bf16/fp16, fp32 accumulation); M <= 256 per launch.

    Schedules: persistent stream-K (default) or, with ``cluster_splits`` = s > 0 (M <= 64), one CTA per
    (tile, K split) with the s CTAs of a tile in a cluster reducing through distributed shared memory.
    ``small_smem`` halves the TMA ring so the next kernel can share the SM (programmatic launch).
    ``w`` is a row-major [N, K] tensor or a PackedWeight (bulk loads of contiguous weight blocks).
    ``swiglu``: w's rows are gate/up interleaved by 64 (`pack_weight(w, interleave=64)`) and out is
    [M, N / 2] = silu(gate) * up, formed in the cluster reduction (a cluster split count of 2, 4, 8 or 16,
    `swiglu_splits`) or, with stream-K and M <= 16, in the epilogue (up rows handed to the gate rows'
    threads through the workspace)."""
    M, N = x.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(M, N // 2 if swiglu else N, dtype=x.dtype, device=x.device)
    st = _state(x.device)
    packed = isinstance(w, PackedWeight)
    wt, pn = (w.data, w.n) if packed else (w, 0)
    if swiglu and (M > 64 or (not cluster_splits and M > 16)):
        raise ValueError("the SwiGLU epilogue needs M <= 64 with the cluster schedule, M <= 16 with stream-K")
    for m0 in range(0, M, 256):
        m1 = min(M, m0 + 256)
        native().gemm(x[m0:m1], wt, out[m0:m1], st["ws"], st["ctr"], st["err"], ctas, pdl, small_smem,
                      cluster_splits if m1 - m0 <= 64 else 0, int(timeout_ms * 1e6), pn, bool(swiglu))
    return out


def cluster_split_count(K: int, splits: int) -> int:
    """CTAs per output tile that the cluster schedule launches for `splits` (K cut into equal shares of
    whole 64-wide k-steps)."""
    kt = (K + BK - 1) // BK
    kps = -(-kt // splits)
    return -(-kt // kps)


def swiglu_splits(K: int, splits: int) -> bool:
    """Whether the SwiGLU epilogue accepts this cluster split count (the launched count divides 64)."""
    s = cluster_split_count(K, splits) if splits > 0 else 0
    return s >= 2 and (BM // 2) % s == 0


def candidates(M: int, N: int, K: int, num_sms: int = 148, swiglu: bool = False) -> list[dict]:
    """Launch configurations worth measuring for one decode shape: stream-K with the full or the half
    ring, and cluster split-K with 2..16 splits while the grid stays within one wave (two CTAs per SM with
    the half ring). With `swiglu` only the schedules the SwiGLU epilogue accepts (stream-K for M <= 16)."""
    cands = [] if swiglu and M > 16 else [dict(), dict(small_smem=True)]
    tiles = (N + 127) // 128
    # the SwiGLU epilogue exists only in the cluster schedule: for wide outputs (more tiles than SMs) its
    # multi-wave grids are measured too, and the caller weighs them against stream-K + the SiLU kernel
    waves = 4 if swiglu else 1
    if M <= 64 and (tiles < num_sms or swiglu):
        for s in (2, 3, 4, 6, 8, 12, 16):
            if s > (K + 63) // 64 or (swiglu and not swiglu_splits(K, s)):
                continue
            if tiles * s <= num_sms * 1.25 * waves and s <= 8:
                cands.append(dict(cluster_splits=s))
            if tiles * s <= num_sms * 2 * waves:
                cands.append(dict(cluster_splits=s, small_smem=True))
    return [dict(c, swiglu=True) for c in cands] if swiglu else cands


_TUNED: dict[tuple, dict] = {}
L2_BYTES = 126 << 20


def _cold_copies(w, budget: int = 2 * L2_BYTES):
    """`w` plus enough random copies that cycling through them exceeds `budget` bytes, so every timed
    launch streams its weights from HBM, as in decode (other layers evict them from L2)."""
    nbytes = w.data.numel() * w.data.element_size() if isinstance(w, PackedWeight) else w.numel() * w.element_size()
    n = max(1, -(-budget // nbytes))
    out = [w]
    for _ in range(n - 1):
        if isinstance(w, PackedWeight):
            out.append(PackedWeight(torch.empty_like(w.data).normal_(0, 0.02), w.n, w.k, w.ranks))
        else:
            out.append(torch.empty_like(w).normal_(0, 0.02))
    return out


def tune(w, M: int, iters: int = 20, swiglu: bool = False) -> dict:
    """Measure every candidate schedule for (M, N, K) the way decode runs it: `iters` back-to-back launches
    captured in one CUDA graph with programmatic dependent launch, cycling through copies of the weight
    that together exceed twice the L2 (weights come from HBM), median of 3 replays; cache the fastest.
    With `swiglu` only schedules with the SwiGLU epilogue; {} when none launches."""
    from .._ext import native as _native

    N, K = w.shape[-2], w.shape[-1]
    key = (M, N, K, w.dtype, w.device.index, isinstance(w, PackedWeight), swiglu)
    if key in _TUNED:
        return _TUNED[key]
    dev = w.device
    x = torch.randn(M, K, device=dev).to(w.dtype)
    y = torch.empty(M, N // 2 if swiglu else N, device=dev, dtype=w.dtype)
    ws = _cold_copies(w)
    C = _native()
    old = C.get_pdl()
    C.set_pdl(True)
    best, best_t = {}, float("inf")
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    try:
        for cand in candidates(M, N, K, sms, swiglu):
            try:
                for i in range(len(ws)):
                    gemm(x, ws[i], y, **cand)
                torch.cuda.synchronize()
            except RuntimeError:
                continue
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in range(iters):
                    gemm(x, ws[i % len(ws)], y, **cand)
            g.replay()
            ts = []
            for _ in range(3):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                g.replay()
                b.record()
                torch.cuda.synchronize()
                ts.append(a.elapsed_time(b) / iters)
            del g
            t = sorted(ts)[1]
            if t < best_t:
                best, best_t = cand, t
    finally:
        C.set_pdl(old)
    _TUNED[key] = dict(best, us=round(best_t * 1000, 2)) if best_t < float("inf") else {}
    del ws
    return _TUNED[key]


def _silu_us(M: int, inter: int, dtype, device, iters: int = 20) -> float:
    """Device time of one SiLU * up launch on [M, 2 inter] (graph of `iters` PDL launches, median of 3)."""
    from ..ops import kernels as K

    C = native()
    gu = torch.randn(M, 2 * inter, device=device).to(dtype)
    out = torch.empty(M, inter, device=device, dtype=dtype)
    old = C.get_pdl()
    C.set_pdl(True)
    try:
        K.silu_mul(gu, out=out)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                K.silu_mul(gu, out=out)
        g.replay()
        ts = []
        for _ in range(3):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) * 1000.0 / iters)
    finally:
        C.set_pdl(old)
    return sorted(ts)[1]


class Linear:
    def __init__(self, weight: torch.Tensor, impl: str = "cob", pdl: bool = False):
        assert impl in ("cob", "torch")
        self.weight, self.impl, self.pdl = weight, impl, pdl
        self.cfg: dict[int, dict] = {}  # batch rows -> tuned launch configuration

    def tune(self, M: int) -> dict:
        if self.impl == "cob" and M not in self.cfg:
            self.cfg[M] = {k: v for k, v in tune(self.weight, M).items() if k != "us"}
        return self.cfg.get(M, {})

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        if self.impl == "torch":
            if out is None:
                return x @ self.weight.t()
            return torch.matmul(x, self.weight.t(), out=out)
        return gemm(x, self.weight, out, pdl=self.pdl, **self.cfg.get(x.shape[0], {}))


class GateUpLinear(Linear):
    """The MLP's gate/up projection followed by SiLU(gate) * up: out [M, I] for x [M, K] and a gate/up weight
    [2I, K]. With this package's GEMMs and a weight packed with `interleave=64`, one launch when a SwiGLU
    epilogue schedule is measured for M (`tune`), else the GEMM (outputs in the interleaved order) and the
    SiLU * up kernel. cuBLAS (`impl="torch"`) or row-major weights: the GEMM and the kernel."""

    def __init__(self, weight, impl: str = "cob", pdl: bool = False):
        super().__init__(weight, impl, pdl)
        self.il = weight.il if isinstance(weight, PackedWeight) else 0
        self.fused: dict[int, dict] = {}  # batch rows -> SwiGLU-epilogue launch configuration
        self._gu: dict[tuple, torch.Tensor] = {}

    def tune(self, M: int) -> dict:
        """The faster of (the best SwiGLU-epilogue launch) and (the best plain launch + the SiLU * up
        kernel), both measured in CUDA graphs with programmatic dependent launch."""
        if self.impl == "cob" and M not in self.fused:
            f = tune(self.weight, M, swiglu=True) if self.il == BM // 2 else {}
            if f:
                plain = tune(self.weight, M)
                if plain and f["us"] > plain["us"] + _silu_us(M, self.weight.shape[0] // 2, self.weight.dtype,
                                                              self.weight.device):
                    f = {}
            self.fused[M] = {k: v for k, v in f.items() if k != "us"}
        if not self.fused.get(M):
            super().tune(M)
        return self.fused.get(M) or self.cfg.get(M, {})

    def kernels(self, M: int) -> int:
        """Kernels one call launches for M rows (as tuned)."""
        return 1 if self.fused.get(M) else 2

    def __call__(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        from ..ops import kernels as K

        M = x.shape[0]
        if out is None:
            out = torch.empty(M, self.weight.shape[0] // 2, dtype=x.dtype, device=x.device)
        if self.fused.get(M):
            return gemm(x, self.weight, out, pdl=self.pdl, **dict(self.fused[M], swiglu=True))
        key = (M, x.device)
        if key not in self._gu:  # allocated once per batch size (before capture: the warm-up step)
            self._gu[key] = torch.empty(M, self.weight.shape[0], dtype=x.dtype, device=x.device)
        super().__call__(x, self._gu[key])
        return K.silu_mul(self._gu[key], out=out, interleave=self.il)
