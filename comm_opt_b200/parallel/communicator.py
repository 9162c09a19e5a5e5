"""Tensor-parallel communicator: the public entry point of the fused decode collective.

    comm = TPCommunicator(group, device=dev, dtype=torch.bfloat16, max_rows=512, max_hidden=8192)
    out, residual = comm.fused_allreduce_add_rmsnorm(x, residual, gamma, eps)

`x` is this rank's partial sum (the row-parallel projection output), `residual` is replicated on
every rank and updated in place to ``residual + sum_ranks(x)``; `out` is
``RMSNorm(residual + sum_ranks(x)) * gamma`` on every rank. The call semantics follow the
reference's fused op (exp/M17_epoch_ab/fused_ar_norm_nf.cu:203-206: x in symmetric memory,
residual/gamma/out local), except that x may be any CUDA tensor and every rank receives the full
new residual.

One kernel per call; the ranks synchronise through the data itself (see csrc/fused_ar.cu), so the
call needs no host barrier and can be captured in CUDA graphs of any grid size and replayed in any
order. Every device-side wait is bounded; a timeout leaves an error word that `check()` turns into
`TPCommTimeout`, after which `reset()` (collective) re-initialises the protocol state.

Emulation: ``TPCommunicator(emulate_world=W, device=dev)`` runs all W ranks in one process on one
GPU; inputs then carry a leading rank dimension ``[W, rows, hidden]`` and every call is a single
kernel launch covering all ranks.
"""
from __future__ import annotations

import os

import torch

from .._ext import native
from .symm import DTYPE_CODE, HeapLayout, SymmetricHeap, plan_layout
from .variant_table import NVLS_VARIANTS, VARIANT_NAMES, VARIANTS, Choice, VariantTable

ERR_BITS = {
    1: "timeout waiting for landing data",
    2: "timeout in flag barrier",
    4: "timeout in NVLS barrier",
    8: "timeout waiting for a row partial",
    16: "bad arguments",
    32: "timeout in all-gather",
    64: "timeout in grid barrier",
    128: "index out of range (checked build; access skipped)",
}


def decode_state(words: list[int], rank: int) -> dict:
    """One rank's control words (int64: epoch, unused | error << 32, err_detail[4]) -> readable state.
    err_detail: [0] = kernel family and phase ((variant << 32) | phase for the fused all-reduce kernels,
    0xF6 << 32 for the fused GEMMs), [1] = where (row << 32 | vector, or the rank's block), [2] = peer
    or block, [3] = the call's epoch."""
    err = (words[1] >> 32) & 0xFFFFFFFF
    d = [w & 0xFFFFFFFFFFFFFFFF for w in words[2:6]]
    fam = d[0] >> 32
    where = dict(kernel="fused_gemm" if fam == 0xF6 else VARIANT_NAMES.get(fam, f"variant {fam}"),
                 phase=d[0] & 0xFFFFFFFF, row=d[1] >> 32, vector=d[1] & 0xFFFFFFFF, peer_or_block=d[2], call=d[3])
    return dict(rank=rank, epoch=words[0], error=err, detail=d, where=where,
                reasons=[m for b, m in ERR_BITS.items() if err & b])


def describe_error(state: dict) -> str:
    w = state["where"]
    return (f"rank {state['rank']}: {', '.join(state['reasons']) or 'no error'} in {w['kernel']} phase {w['phase']} "
            f"(row {w['row']}, vector {w['vector']}, peer/block {w['peer_or_block']}, call {w['call']}; "
            f"epoch now {state['epoch']})")


class TPCommError(RuntimeError):
    pass


class TPCommTimeout(TPCommError):
    pass


def default_timeout_ms() -> float:
    return float(os.environ.get("COB_WAIT_TIMEOUT_MS", "1000"))


def _weight_operand(w):
    """(tensor handed to the kernel, output features N, packed?) of a row-major or packed weight."""
    from ..models.gemm import PackedWeight

    if isinstance(w, PackedWeight):
        return w.data, w.n, True
    return w, w.shape[-2], False


class TPCommunicator:
    def __init__(self, group=None, *, emulate_world: int | None = None, device=None, dtype=torch.bfloat16,
                 max_rows: int = 512, max_hidden: int = 8192, max_gather: int = 4096,
                 timeout_ms: float | None = None, pdl: bool = True, table: VariantTable | None = None,
                 allow_nvls: bool = True, backend: str = "symm_mem"):
        import torch.distributed as dist

        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        self.esize = torch.tensor([], dtype=dtype).element_size()
        self.max_rows = max_rows
        self.max_hidden = max_hidden
        self.timeout_ns = int((timeout_ms if timeout_ms is not None else default_timeout_ms()) * 1e6)
        self.pdl = pdl
        self.table = table if table is not None else VariantTable.load()
        self.group = group
        self.emulated = emulate_world is not None
        if self.emulated:
            self.world, self.rank = int(emulate_world), 0
        elif group is not None or (dist.is_available() and dist.is_initialized()):
            self.group = group if group is not None else dist.group.WORLD
            self.world, self.rank = dist.get_world_size(self.group), dist.get_rank(self.group)
        else:
            self.world, self.rank = 1, 0
        self.heap: SymmetricHeap | None = None
        self.layout: HeapLayout | None = None
        if self.world > 1:
            self.layout = plan_layout(self.world, max_rows, max_hidden, self.esize, max_gather)
            if self.emulated:
                self.heap = SymmetricHeap.emulated(self.world, self.layout, self.device)
            elif backend == "ipc":
                self.heap = SymmetricHeap.from_group_ipc(self.group, self.layout, self.device)
            else:
                self.heap = SymmetricHeap.from_group(self.group, self.layout, self.device)
            self._layout_list = self.layout.as_list()
            self._init_state()
        self.have_nvls = bool(self.heap and self.heap.mc and allow_nvls)
        self.last_choice: Choice | None = None
        self.stamps: torch.Tensor | None = None
        self._fg: dict[int, dict] = {}  # layer-boundary fused GEMM workspaces by inner size K
        self._fg_err_t: torch.Tensor | None = None
        self.last_fused_gemm: tuple | None = None

    @classmethod
    def from_config(cls, group=None, config=None, **kw) -> "TPCommunicator":
        """Build from a CommConfig (defaults + COB_* environment overrides when `config` is None)."""
        from .config import CommConfig

        cfg = config if config is not None else CommConfig.from_env()
        return cls(group, **cfg.kwargs(), **kw)

    # ------------------------------------------------------------------ state management
    def _host_barrier(self):
        if not self.emulated and self.world > 1:
            import torch.distributed as dist

            dist.barrier(group=self.group, device_ids=[self.device.index]) if dist.get_backend(
                self.group) == "nccl" else dist.barrier(group=self.group)

    def _init_state(self):
        with torch.cuda.device(self.device):
            for h in self.heap.local_heaps():
                native().init_heap(h, self._layout_list, DTYPE_CODE[self.dtype])
            torch.cuda.synchronize(self.device)
        self._host_barrier()

    def reset(self):
        """Collective: re-initialise flags, epochs and landing buffers on every rank (after an error)."""
        if self.world == 1:
            return
        torch.cuda.synchronize(self.device)
        self._host_barrier()
        for ws in self._fg.values():
            ws["flags"].zero_()
        self._init_state()

    def error_state(self) -> list[dict]:
        """Synchronises and reads the error word of each local rank."""
        if self.world == 1:
            return []
        torch.cuda.synchronize(self.device)
        return [decode_state(self.heap.state_words(h).cpu().tolist(), r if self.emulated else self.rank)
                for r, h in enumerate(self.heap.local_heaps())]

    def epochs(self) -> list[int]:
        return [s["epoch"] for s in self.error_state()]

    def check(self):
        """Raise TPCommTimeout if any local rank recorded a bounded-wait timeout."""
        for s in self.error_state():
            if s["error"]:
                raise TPCommTimeout(describe_error(s) + "; call reset() on every rank before reuse")

    # ------------------------------------------------------------------ variant choice
    def choose(self, rows: int, hidden: int, variant="auto", blocks=0, threads=0, cluster=0) -> Choice:
        if variant in (None, "auto", 0):
            c = self.table.lookup(self.world, self.dtype, self.esize, hidden, rows, self.have_nvls)
            c = Choice(c.variant, blocks or c.blocks, threads or c.threads, cluster or c.cluster, c.p50_us)
        else:
            v = VARIANTS[variant] if isinstance(variant, str) else int(variant)
            if v in NVLS_VARIANTS and not self.have_nvls:
                raise TPCommError(f"{VARIANT_NAMES[v]} needs NVSwitch multicast, not available here")
            c = Choice(v, blocks, threads, cluster)
        return c

    # ------------------------------------------------------------------ phase stamps
    PHASES = ("start", "sent", "reduced", "received", "done")

    def enable_stamps(self, cap: int = 2048):
        """Record %globaltimer at every phase boundary of every block of every call (ring of `cap` calls)."""
        ranks = self.world if self.emulated else 1
        self.stamps = torch.zeros(ranks, cap, native().kMaxBlocks, native().kStampPhases, dtype=torch.int64,
                                  device=self.device)

    def disable_stamps(self):
        self.stamps = None

    def stamp_summary(self, epochs: list[int], blocks: int) -> dict:
        """Per phase, mean over the given calls of (latest block's stamp - earliest block's start) in us,
        per local rank: the critical path of the call split into phases."""
        st = self.stamps.cpu()
        cap = st.shape[1]
        out = {}
        for r in range(st.shape[0]):
            acc = {ph: 0.0 for ph in self.PHASES[1:]}
            for e in epochs:
                blk = st[r, e % cap, :blocks]
                t0 = int(blk[:, 0].min())
                for i, ph in enumerate(self.PHASES[1:], start=1):
                    acc[ph] += (int(blk[:, i].max()) - t0) / 1000.0 / len(epochs)
            out[r] = acc
        return out

    # ------------------------------------------------------------------ ops
    def _shape(self, x: torch.Tensor) -> tuple[int, int]:
        hidden = x.shape[-1]
        if self.emulated:
            assert x.shape[0] == self.world, "emulated inputs are [world, rows, hidden]"
            rows = x[0].numel() // hidden
        else:
            rows = x.numel() // hidden
        if rows > self.max_rows or hidden > self.max_hidden:
            raise TPCommError(f"[{rows}, {hidden}] exceeds the communicator capacity "
                              f"[{self.max_rows}, {self.max_hidden}]")
        return rows, hidden

    def _launch(self, x, residual, gamma, out, eps, norm, variant, blocks, threads, cluster, dry_run=False):
        rows, hidden = self._shape(x)
        if x.dtype != self.dtype:
            raise TPCommError(f"communicator dtype is {self.dtype}, got {x.dtype}")
        c = self.choose(rows, hidden, variant, blocks, threads, cluster)
        stride = rows * hidden if self.emulated else 0
        with torch.cuda.device(self.device):
            rc, v, b, t, cl = native().fused_ar(
                self.heap.bases, self.heap.mc, self._layout_list, x, residual if norm else x,
                gamma if norm else x, out, self.rank, rows, hidden, float(eps), c.variant, c.blocks, c.threads,
                c.cluster, int(self.emulated), int(self.pdl), int(norm), self.timeout_ns, stride, stride, stride,
                dry_run, self.stamps)
        if rc != 0:
            raise TPCommError(f"fused_ar: unsupported configuration {VARIANT_NAMES.get(v, v)} rows={rows} "
                              f"hidden={hidden} world={self.world} blocks={b} threads={t} cluster={cl} "
                              f"(cuda status {rc})")
        self.last_choice = Choice(v, b, t, cl, c.p50_us)
        return self.last_choice

    def fused_allreduce_add_rmsnorm(self, x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor,
                                    eps: float = 1e-6, out: torch.Tensor | None = None, variant="auto",
                                    blocks: int = 0, threads: int = 0, cluster: int = 0):
        """Returns (out, residual); residual is updated in place."""
        if out is None:
            out = torch.empty_like(x)
        if self.world == 1:
            native().add_rmsnorm(x, residual, gamma, out, float(eps))
            return out, residual
        self._launch(x, residual, gamma, out, eps, 1, variant, blocks, threads, cluster)
        return out, residual

    def all_reduce(self, x: torch.Tensor, out: torch.Tensor | None = None, variant="auto", blocks: int = 0,
                   threads: int = 0, cluster: int = 0) -> torch.Tensor:
        """Plain sum over ranks (same kernels with the residual/norm epilogue switched off)."""
        if out is None:
            out = torch.empty_like(x)
        if self.world == 1:
            out.copy_(x)
            return out
        self._launch(x, None, None, out, 0.0, 0, variant, blocks, threads, cluster)
        return out

    def all_gather_u32(self, inp: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Gather a small int32/uint32/float32 vector from every rank: out [world, n]."""
        n = inp.shape[-1]
        if out is None:
            out = torch.empty((self.world, n) if not self.emulated else (self.world, self.world, n),
                              dtype=inp.dtype, device=inp.device)
        if self.world == 1:
            out.view(-1).copy_(inp.view(-1))
            return out
        with torch.cuda.device(self.device):
            native().allgather_u32(self.heap.bases, self._layout_list, inp, out, self.rank, n, int(self.emulated),
                                   self.timeout_ns, n if self.emulated else 0, self.world * n if self.emulated else 0)
        return out

    # ------------------------------------------------------------------ layer-boundary fused GEMMs
    def _fg_workspace(self, K: int) -> dict:
        ws = self._fg.get(K)
        if ws is None:
            ranks = self.world if self.emulated else 1
            n = native().kMaxPieces
            ws = dict(act=torch.zeros(ranks * self.max_rows, K, dtype=torch.bfloat16, device=self.device),
                      flags=torch.zeros(ranks, n, dtype=torch.int32, device=self.device),
                      pss=torch.zeros(ranks, n, self.max_rows, dtype=torch.float32, device=self.device))
            self._fg[K] = ws
        return ws

    def prepare_fused_gemm(self, K: int):
        """Allocate the workspace of ar_norm_gemm for inner size K (call before CUDA-graph capture)."""
        self._fg_workspace(K)

    def _fg_dims(self, t: torch.Tensor) -> tuple[int, int]:
        if self.emulated:
            assert t.shape[0] == self.world, "emulated operands are [world, rows, cols]"
            return t[0].numel() // t.shape[-1], t.shape[-1]
        return t.numel() // t.shape[-1], t.shape[-1]

    def gemm_push(self, x: torch.Tensor, w, splits: int = 0, dry_run: bool = False):
        """Row-parallel GEMM whose epilogue is the first half of the all-reduce: x [M, K] @ w[N, K]^T is
        pushed (bf16) into every rank's landing buffers; `ar_norm_gemm` (or nothing else) must follow.
        Emulation: x [W, M, K], w [W, N, K]. `w` may be a PackedWeight (models.gemm.pack_weight)."""
        if self.world == 1 or self.dtype != torch.bfloat16:
            raise TPCommError("fused GEMMs need world > 1 and a bf16 communicator")
        M, K = self._fg_dims(x)
        wt, N, packed = _weight_operand(w)
        if M > self.max_rows or N > self.max_hidden:
            raise TPCommError(f"gemm_push [{M}, {N}] exceeds the communicator capacity")
        with torch.cuda.device(self.device):
            plan = native().fused_gemm(0, self.heap.bases, self._layout_list, wt, x=x, err=self._fg_err(),
                                       rank=self.rank, M=M, N=N, K=K, eps=0.0, emulate=int(self.emulated), splits=splits,
                                       pdl=int(self.pdl), timeout_ns=self.timeout_ns, res_rs=0, dry_run=dry_run,
                                       packed=packed)
        self.last_fused_gemm = ("gemm_push", tuple(plan))
        return plan

    def _fg_err(self) -> torch.Tensor:
        if self._fg_err_t is None:
            self._fg_err_t = torch.zeros(1, dtype=torch.int32, device=self.device)
        return self._fg_err_t

    EPILOGUES = {"plain": 0, "swiglu": 1, "rope_kv": 2}

    @staticmethod
    def interleave_gate_up(w: torch.Tensor) -> torch.Tensor:
        """[..., 2I, K] = [gate rows; up rows] -> the swiglu epilogue's layout: output tile t (128 rows)
        holds gate rows 64t..64t+63 then the matching up rows (I % 64 == 0)."""
        I2, K = w.shape[-2], w.shape[-1]
        I = I2 // 2
        assert I % 64 == 0, "intermediate size must be a multiple of 64"
        lead = w.shape[:-2]
        g = w[..., :I, :].reshape(*lead, I // 64, 64, K)
        u = w[..., I:, :].reshape(*lead, I // 64, 64, K)
        return torch.stack([g, u], dim=-3).reshape(*lead, I2, K).contiguous()

    def ar_norm_gemm(self, residual: torch.Tensor, gamma: torch.Tensor, w, eps: float = 1e-6,
                     out: torch.Tensor | None = None, splits: int = 0, dry_run: bool = False,
                     epilogue: str = "plain", rope: dict | None = None) -> torch.Tensor:
        """Second half of the all-reduce fused with RMSNorm and the next column-parallel GEMM:
        h = residual + sum_ranks(pushed partials) (residual updated in place), z = (RMSNorm(h) * gamma) @ w^T.
        epilogue "plain": out = z [M, N]. "swiglu": w tile-interleaved (`interleave_gate_up`), out = silu(gate)
        * up [M, N / 2]. "rope_kv": z holds [q heads | k heads | v heads] of 128; out = RoPE(q) [M, nq, 128],
        RoPE(k) and v written into the paged caches at rope["positions"] (keys: positions, cos, sin,
        block_tables, k_cache, v_cache, nq, nkv). Emulation: residual [W, M, K], w [W, N, K]. `w` may be a
        PackedWeight (models.gemm.pack_weight)."""
        if self.world == 1 or self.dtype != torch.bfloat16:
            raise TPCommError("fused GEMMs need world > 1 and a bf16 communicator")
        M, K = self._fg_dims(residual)
        wt, N, packed = _weight_operand(w)
        epi = self.EPILOGUES[epilogue]
        if M > self.max_rows or K > self.max_hidden:
            raise TPCommError(f"ar_norm_gemm [{M}, {K}] exceeds the communicator capacity")
        if out is None and not dry_run:
            cols = N // 2 if epi == 1 else (rope["nq"] * 128 if epi == 2 else N)
            shape = (self.world, M, cols) if self.emulated else (M, cols)
            out = torch.empty(shape, dtype=torch.bfloat16, device=residual.device)
        ws = self._fg_workspace(K)
        r = rope or {}
        with torch.cuda.device(self.device):
            plan = native().fused_gemm(1, self.heap.bases, self._layout_list, wt, residual=residual, gamma=gamma,
                                       y=out if out is not None else residual, act=ws["act"], flags=ws["flags"],
                                       pss=ws["pss"], err=self._fg_err(), rank=self.rank, M=M, N=N, K=K,
                                       eps=float(eps), emulate=int(self.emulated), splits=splits,
                                       pdl=int(self.pdl), timeout_ns=self.timeout_ns,
                                       res_rs=M * K if self.emulated else 0, dry_run=dry_run, epi=epi,
                                       positions=r.get("positions"), cos=r.get("cos"), sin=r.get("sin"),
                                       block_tables=r.get("block_tables"), k_cache=r.get("k_cache"),
                                       v_cache=r.get("v_cache"), nq=r.get("nq", 0), nkv=r.get("nkv", 0),
                                       packed=packed)
        self.last_fused_gemm = ("ar_norm_gemm", tuple(plan))
        return out

    def fused_epilogue_supported(self, M: int, N: int, K: int, epilogue: str) -> bool:
        """Whether ar_norm_gemm can run this epilogue for [M, K] x [N, K]^T (a plan with 2..8 splits)."""
        ranks = self.world if self.emulated else 1
        dummy_w = torch.empty(ranks * N, K, dtype=torch.bfloat16, device=self.device)
        dummy_r = torch.empty((ranks, M, K) if self.emulated else (M, K), dtype=torch.bfloat16, device=self.device)
        self.ar_norm_gemm(dummy_r, dummy_r.new_empty(K), dummy_w, dry_run=True, epilogue=epilogue)
        return self.last_fused_gemm[1][2] > 0

    def close(self):
        """Collective teardown: every rank unmaps its peers' heaps before any heap is freed."""
        if self.heap is None:
            return
        torch.cuda.synchronize(self.device)
        self._host_barrier()
        if hasattr(self.heap, "close_ipc"):
            self.heap.close_ipc()
        self._host_barrier()
        self.heap = None

    def describe(self) -> dict:
        return dict(world=self.world, rank=self.rank, emulated=self.emulated, dtype=str(self.dtype),
                    max_rows=self.max_rows, max_hidden=self.max_hidden, nvls=self.have_nvls,
                    heap_bytes=self.layout.total if self.layout else 0, timeout_ms=self.timeout_ns / 1e6)
