"""Implementations compared by the fused-op sweep (the reference's headline fused-op benchmark), behind one interface.

Every implementation turns (x, residual, gamma, eps) of this rank into a zero-argument callable that
performs ONE fused all-reduce + residual add + RMSNorm on static buffers, so K calls can be captured
in a CUDA graph and replayed (the reference's timing method, exp/M17_epoch_ab/bench_ab.py:167-195).

  ours:<variant>     TPCommunicator.fused_allreduce_add_rmsnorm (lamport_1s/2s, pull_1s/2s, nvls_1s/2s, auto)
  ours_ipc:<variant> the same on a CUDA-IPC heap instead of a multicast-capable symmetric-memory heap
  ours_pdl:<variant> the same with programmatic dependent launch between consecutive calls
  nccl_norm          NCCL all-reduce (in place) + vLLM fused_add_rms_norm  (reference U_nccl,
                     exp/M9_fused_baselines/bench_fused.py:88-89)
  vllm_car           vLLM custom all-reduce + fused_add_rms_norm           (reference U_vllm,
                     exp/M17_epoch_ab/bench_ab.py:117-120)
  trt_oneshot/twoshot FlashInfer TRT-LLM allreduce_fusion kARResidualRMSNorm, native sm_100 build
                     (reference F_trt_one/two, exp/M17_epoch_ab/bench_ab.py:107-114)
  ref_m16nf          the reference's own prototype kernel (exp/M17_epoch_ab/fused_ar_norm_nf.cu,
                     unmodified source from the reference tree, built for sm_100a; 8 ranks only,
                     residual kept sharded by rows as in the reference)
"""
from __future__ import annotations

import contextlib
import math
import os
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[2]
# Prebuilt JIT baselines live under <repo>/baseline; COB_ROOT lets a run name the repository by the
# same path it was built under, so the JIT builders find their outputs up to date.
BASE = Path(os.environ.get("COB_ROOT", str(ROOT))) / "baseline"


class Impl:
    name = "?"
    residual_rows = "all"  # rows of the residual the implementation updates ("all" or "own")

    def capture_ctx(self):
        return contextlib.nullcontext()

    def available(self, rows: int, hidden: int) -> str:
        """'' if the size is supported, else the reason it is skipped."""
        return ""

    def make(self, x, residual, gamma, eps):
        raise NotImplementedError

    def close(self):
        pass


class Ours(Impl):
    def __init__(self, comm, variant="auto"):
        self.comm, self.variant = comm, variant
        self.name = f"ours:{variant}"

    def available(self, rows, hidden):
        from ..parallel.variant_table import NVLS_VARIANTS, VARIANTS

        if self.variant != "auto" and VARIANTS[self.variant] in NVLS_VARIANTS and not self.comm.have_nvls:
            return "no NVSwitch multicast"
        if self.variant in ("lamport_2s", "pull_2s", "nvls_2s"):
            hv = hidden * self.comm.esize // 16
            if hv % self.comm.world or hv % 32:
                return "hidden not divisible for two-shot"
        return ""

    pdl = False
    owns_comm = False  # close the communicator with this implementation (the IPC-heap one)

    def close(self):
        if self.owns_comm:
            self.comm.close()

    def make(self, x, residual, gamma, eps):
        out = torch.empty_like(x)
        comm, v, pdl = self.comm, self.variant, self.pdl

        def fn():
            old = comm.pdl
            comm.pdl = pdl or old
            try:
                comm.fused_allreduce_add_rmsnorm(x, residual, gamma, eps, out=out, variant=v)
            finally:
                comm.pdl = old
            return out

        return fn


def _vllm_ops():
    import vllm._custom_ops  # noqa: F401  registers torch.ops._C

    return torch.ops._C


class NcclNorm(Impl):
    name = "nccl_norm"

    def __init__(self, group=None):
        self.group = group
        try:
            self.C = _vllm_ops()
        except Exception:  # pragma: no cover - vLLM missing: the norm falls back to this package's kernel
            self.C = None
            self.name = "nccl_cobnorm"  # rows say which norm kernel the baseline ran

    def make(self, x, residual, gamma, eps):
        C, group = self.C, self.group

        def fn():
            dist.all_reduce(x, group=group)
            if C is not None:
                C.fused_add_rms_norm(x, residual, gamma, eps)
            else:
                from ..ops.kernels import add_rmsnorm

                add_rmsnorm(x, residual, gamma, eps, out=x)
            return x

        return fn


class VllmCar(Impl):
    name = "vllm_car"

    def __init__(self, cpu_group, device, max_bytes):
        from vllm.distributed.device_communicators.custom_all_reduce import CustomAllreduce

        self.C = _vllm_ops()
        self.car = CustomAllreduce(cpu_group, device, max_size=max_bytes)
        if self.car.disabled:
            raise RuntimeError("vLLM custom all-reduce is disabled on this system")

    def available(self, rows, hidden):
        return "" if self.car.should_custom_ar(torch.empty(rows * hidden, dtype=torch.bfloat16,
                                                           device="cuda")) else "vLLM declines this size"

    def capture_ctx(self):
        return self.car.capture()

    def make(self, x, residual, gamma, eps):
        car, C = self.car, self.C

        def fn():
            out = car.custom_all_reduce(x)
            C.fused_add_rms_norm(out, residual, gamma, eps)
            return out

        return fn

    def close(self):
        self.car.close()


class FlashInferTrt(Impl):
    def __init__(self, rank, world, max_rows, hidden, cpu_group, oneshot: bool):
        os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", str(BASE / "_flashinfer"))
        import flashinfer.comm.trtllm_ar as fi

        self.fi, self.rank, self.world, self.oneshot = fi, rank, world, oneshot
        self.name = "trt_oneshot" if oneshot else "trt_twoshot"
        self.handles, self.ws = fi.trtllm_create_ipc_workspace_for_all_reduce_fusion(rank, world, max_rows, hidden,
                                                                                      group=cpu_group)[:2]
        self.cpu_group = cpu_group

    def available(self, rows, hidden):
        if not self.oneshot and rows <= self.world:
            return "two-shot needs tokens > world size (FlashInfer assertion)"
        return ""

    def make(self, x, residual, gamma, eps):
        fi, out = self.fi, torch.empty_like(x)
        T, H = x.shape

        def fn():
            fi.trtllm_allreduce_fusion(
                allreduce_in=x, world_size=self.world, world_rank=self.rank, token_num=T, hidden_dim=H,
                workspace_ptrs=self.ws, launch_with_pdl=False, trigger_completion_at_end=True, fp32_acc=True,
                pattern_code=fi.AllReduceFusionPattern.kARResidualRMSNorm, use_oneshot=self.oneshot,
                allreduce_out=None, residual_in=residual, residual_out=residual, norm_out=out, quant_out=None,
                scale_out=None, rms_gamma=gamma, rms_eps=eps, scale_factor=None, layout_code=None)
            return out

        return fn

    def close(self):
        self.fi.trtllm_destroy_ipc_workspace_for_all_reduce_fusion(self.handles, group=self.cpu_group)


class RefProto(Impl):
    """The reference prototype, unmodified source (copied into baseline/_ref/), JIT-built for sm_100a."""

    name = "ref_m16nf"
    residual_rows = "own"

    def __init__(self, rank, world, max_rows, hidden, dtype, device, ctas=64):
        import torch.distributed._symmetric_memory as symm_mem
        from torch.utils.cpp_extension import load

        if world != 8:
            raise RuntimeError("the reference prototype is hard-wired to 8 ranks")
        src = BASE / "_ref" / "exp" / "M17_epoch_ab" / "fused_ar_norm_nf.cu"
        if not src.exists():
            raise RuntimeError(f"reference source not present at {src}")
        bdir = BASE / "_ref_build"
        bdir.mkdir(parents=True, exist_ok=True)
        self.ext = load(name="ref_m17nf_fused_ar_norm", sources=[str(src)],
                        extra_cuda_cflags=["-O3", "-gencode=arch=compute_100a,code=sm_100a"],
                        build_directory=str(bdir), verbose=False)
        self.rank, self.world, self.H, self.ctas = rank, world, hidden, ctas
        self.gpr = math.ceil(math.ceil(hidden / 4 / 15) / 4)
        rows_per = math.ceil(max_rows / world)
        self.x_buf = symm_mem.empty(max_rows * hidden, dtype=dtype, device=device)
        self.land = symm_mem.empty(2 * world * rows_per * self.gpr * 64, dtype=torch.int64, device=device)
        self.flags = symm_mem.empty(128 * world, dtype=torch.int32, device=device)
        g = dist.group.WORLD
        self.x_ptrs = list(symm_mem.rendezvous(self.x_buf, g).buffer_ptrs)
        self.land_ptrs = list(symm_mem.rendezvous(self.land, g).buffer_ptrs)
        self.flag_ptrs = list(symm_mem.rendezvous(self.flags, g).buffer_ptrs)
        self.ctr = torch.zeros(128, dtype=torch.int64, device=device)
        self.reset()

    def reset(self):
        torch.cuda.synchronize()
        dist.barrier()
        self.land.zero_()
        self.flags.zero_()
        self.ctr.zero_()
        torch.cuda.synchronize()
        dist.barrier()

    def make(self, x, residual, gamma, eps):
        T, H = x.shape
        self.x_buf[:T * H].copy_(x.view(-1))
        self.reset()
        out = torch.empty_like(x)
        rp = math.ceil(T / self.world)

        def fn():
            self.ext.fused_ar_norm(self.x_ptrs, self.land_ptrs, self.flag_ptrs, self.ctr, residual, gamma, out,
                                   self.rank, T, H, eps, self.ctas, rp, self.gpr)
            return out

        return fn


def build(names: list[str], *, comm, rank, world, max_rows, hidden, dtype, device, cpu_group) -> tuple[list, dict]:
    """Instantiate the requested implementations; returns (impls, {name: reason} for unavailable ones)."""
    impls, skipped = [], {}
    comm_ipc = None
    for n in names:
        try:
            if n.startswith("ours:"):
                impls.append(Ours(comm, n.split(":", 1)[1]))
            elif n.startswith("ours_ipc:"):
                # the same kernels on a heap shared by CUDA IPC (no multicast object bound to it)
                if comm_ipc is None:
                    from ..parallel import TPCommunicator

                    comm_ipc = TPCommunicator(comm.group, device=device, dtype=dtype, max_rows=max_rows,
                                              max_hidden=hidden, backend="ipc", pdl=comm.pdl)
                o = Ours(comm_ipc, n.split(":", 1)[1])
                o.name = n
                o.owns_comm = not any(getattr(i, "owns_comm", False) for i in impls)
                impls.append(o)
            elif n.startswith("ours_pdl:"):
                o = Ours(comm, n.split(":", 1)[1])
                o.name, o.pdl = n, True
                impls.append(o)
            elif n == "nccl_norm":
                impls.append(NcclNorm())
            elif n == "vllm_car":
                impls.append(VllmCar(cpu_group, device, max_rows * hidden * 2))
            elif n in ("trt_oneshot", "trt_twoshot"):
                impls.append(FlashInferTrt(rank, world, max_rows, hidden, cpu_group, n == "trt_oneshot"))
            elif n == "ref_m16nf":
                impls.append(RefProto(rank, world, max_rows, hidden, dtype, device))
            else:
                skipped[n] = "unknown implementation"
        except Exception as e:  # record and continue: a baseline that cannot run here is reported as such
            skipped[n] = f"{type(e).__name__}: {str(e)[:300]}"
    return impls, skipped
