"""Symmetric heap: one device allocation per rank, mapped by every peer (and multicast-bound).

All buffers of the fused all-reduce family sit at the same byte offset in every rank's heap
(layout planned by ``plan_layout``), so device code reaches buffer B of rank r at
``bases[r] + layout.B`` and the NVSwitch-reduced view at ``mc + layout.B``.

Two back ends:

* ``SymmetricHeap.from_group`` - one process per GPU; the heap comes from PyTorch symmetric
  memory (``torch.distributed._symmetric_memory``: cuMem allocation, peer mapping and, when the
  NVSwitch supports it, a multicast object), exchanged over the process group. The reference
  allocates its prototype buffers the same way (exp/M17_epoch_ab/bench_ab.py:78-86).
* ``SymmetricHeap.from_group_ipc`` - one process per GPU; our own heap (cudaMalloc) shared through
  CUDA IPC handles exchanged over the process group: plain NVLink peer mappings, never bound to a
  multicast object (used where NVLS must stay off, e.g. fault-injection tests).
* ``SymmetricHeap.emulated`` - all ranks on ONE GPU: ``world`` separate regions of one allocation,
  used to run the whole multi-rank protocol inside a single kernel launch on one GPU.
"""
from __future__ import annotations

from dataclasses import astuple, dataclass

import torch

from .._ext import available, native

FIELDS = ("state", "flags", "nvls", "land1", "rs", "ag", "agp", "stage", "hbuf", "hpart", "gather", "total",
          "world", "max_rows", "max_hv", "sv_max", "esize", "max_gather")

MAX_BLOCKS = 296        # per-block barrier slots and epoch words (two CTAs on each of 148 SMs)
MAX_WORLD = 8
RANK_STATE_BYTES = 6144  # sizeof(cob::RankState)


@dataclass(frozen=True)
class HeapLayout:
    state: int
    flags: int
    nvls: int
    land1: int
    rs: int
    ag: int
    agp: int
    stage: int
    hbuf: int
    hpart: int
    gather: int
    total: int
    world: int
    max_rows: int
    max_hv: int
    sv_max: int
    esize: int
    max_gather: int

    def as_list(self) -> list[int]:
        return list(astuple(self))


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def plan_layout_py(world: int, max_rows: int, max_hidden: int, esize: int, max_gather: int) -> HeapLayout:
    """Pure-Python statement of the native ``plan_layout`` (kept identical; a test compares them)."""
    max_hv = max_hidden * esize // 16
    sv_max = (max_hv + world - 1) // world
    off = 0
    out = {}

    def take(name, nbytes):
        nonlocal off
        out[name] = off
        off = _align(off + nbytes, 4096)

    R, W, HV, SV = max_rows, world, max_hv, sv_max
    take("state", RANK_STATE_BYTES)
    take("flags", MAX_BLOCKS * MAX_WORLD * 8)
    take("nvls", MAX_BLOCKS * 2 * 4)
    take("land1", 2 * W * R * HV * 16)
    take("rs", 2 * W * R * SV * 16)
    take("ag", 2 * W * R * SV * 16)
    pu = (SV + 31) // 32  # partial-sum units per owner slice (32 vectors each)
    take("agp", 2 * W * R * pu * 8)
    take("stage", 2 * R * HV * 16)
    take("hbuf", R * HV * 16)
    take("hpart", R * W * pu * 8)
    take("gather", 2 * W * max_gather * 8)
    total = _align(off, 2 << 20)
    return HeapLayout(total=total, world=world, max_rows=max_rows, max_hv=max_hv, sv_max=sv_max, esize=esize,
                      max_gather=max_gather, **out)


def plan_layout(world: int, max_rows: int, max_hidden: int, esize: int, max_gather: int = 4096) -> HeapLayout:
    if available():
        return HeapLayout(*native().plan_layout(world, max_rows, max_hidden, esize, max_gather))
    return plan_layout_py(world, max_rows, max_hidden, esize, max_gather)


DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


class SymmetricHeap:
    """Per-rank heap pointers plus the local allocation that owns them."""

    def __init__(self, layout: HeapLayout, bases: list[int], mc: int, tensor: torch.Tensor, rank: int,
                 emulated: bool, handle=None):
        self.layout = layout
        self.bases = [int(b) for b in bases]
        self.mc = int(mc)
        self.tensor = tensor  # uint8; emulated: [world * total], real: [total]
        self.rank = rank
        self.world = layout.world
        self.emulated = emulated
        self.handle = handle

    @classmethod
    def from_group(cls, group, layout: HeapLayout, device: torch.device) -> "SymmetricHeap":
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        t = symm_mem.empty(layout.total, dtype=torch.uint8, device=device)
        hdl = symm_mem.rendezvous(t, group)
        rank = dist.get_rank(group)
        ptrs = [int(p) for p in hdl.buffer_ptrs]
        off = t.data_ptr() - ptrs[rank]  # the tensor may sit at an offset inside the symmetric allocation
        try:
            mc = int(hdl.multicast_ptr or 0)
        except (RuntimeError, AttributeError):  # no NVSwitch multicast on this system
            mc = 0
        return cls(layout, [p + off for p in ptrs], mc + off if mc else 0, t, rank, emulated=False, handle=hdl)

    @classmethod
    def from_group_ipc(cls, group, layout: HeapLayout, device: torch.device) -> "SymmetricHeap":
        import torch.distributed as dist

        C = native()
        idx = torch.device(device).index
        t = C.ipc_alloc(layout.total, idx)
        handles = [None] * dist.get_world_size(group)
        dist.all_gather_object(handles, C.ipc_handle(t), group=group)
        rank = dist.get_rank(group)
        bases = [t.data_ptr() if r == rank else C.ipc_open(h, idx) for r, h in enumerate(handles)]
        heap = cls(layout, bases, 0, t, rank, emulated=False)
        heap.opened = [b for r, b in enumerate(bases) if r != rank]
        heap.device_index = idx
        return heap

    def close_ipc(self):
        """Unmap peers' heaps (collective use: call on every rank, then barrier, before freeing)."""
        for b in getattr(self, "opened", []):
            native().ipc_close(b, self.device_index)
        self.opened = []

    @classmethod
    def emulated(cls, world: int, layout: HeapLayout, device: torch.device) -> "SymmetricHeap":
        t = torch.empty(world * layout.total, dtype=torch.uint8, device=device)
        base = t.data_ptr()
        return cls(layout, [base + r * layout.total for r in range(world)], 0, t, 0, emulated=True)

    def local_heaps(self) -> list[torch.Tensor]:
        """Heaps this process owns (all of them when emulated)."""
        if self.emulated:
            return [self.tensor[r * self.layout.total:(r + 1) * self.layout.total] for r in range(self.world)]
        return [self.tensor]

    def state_words(self, heap: torch.Tensor) -> torch.Tensor:
        """int64 view of the first 48 bytes of a RankState: epoch, (unused|error<<32), err_detail[4]."""
        return heap[self.layout.state:self.layout.state + 48].view(torch.int64)
