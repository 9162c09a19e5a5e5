"""Residency of the layer-boundary consumer GEMM, checked without a GPU.

The consumer GEMM (`k_ar_norm_gemm`, comm_opt_b200/csrc/fused_gemm.cu) folds the all-reduce +
residual + RMSNorm into the next GEMM: its CTAs wait for all-reduce pieces that other CTAs of the same
launch produce, so the whole grid must be resident at once. `launch_ar_norm_gemm` admits grids of up
to two CTAs per SM for tiles of 16..64 batch rows (and the host planner sizes the gate_up consumer at
224 CTAs on 148 SMs). This test checks, from the compiler's `-Xptxas -v` resources and the planner's
dynamic shared memory, that two such CTAs fit one sm_100a SM: registers (allocated per warp in units
of 256), shared memory (plus the 1 KB the hardware reserves per CTA) and tensor memory columns.
"""
import re
import shutil

import pytest

SM_REGS = 65536
REG_UNIT = 256
SM_SMEM = 228 * 1024
CTA_RESERVED_SMEM = 1024
TMEM_COLS = 512
THREADS = 192  # kThreads of fused_gemm.cu


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not found")
def test_consumer_gemm_two_ctas_per_sm():
    from comm_opt_b200._ext import native
    from comm_opt_b200.harness.ptxas_report import report

    rows = report(["fused_gemm.cu"], r"k_ar_norm_gemm<(16|32|64), true>")
    assert sorted(int(re.search(r"<(\d+),", r["kernel"]).group(1)) for r in rows) == [16, 32, 64]
    C = native()
    for r in rows:
        bn = int(re.search(r"<(\d+),", r["kernel"]).group(1))
        regs_per_warp = -(-r["regs"] * 32 // REG_UNIT) * REG_UNIT
        assert 2 * regs_per_warp * (THREADS // 32) <= SM_REGS, (r["kernel"], r["regs"])
        # a batch of bn rows gets tiles of bn batch rows; the planner's dynamic shared memory
        bn_plan, *_, smem = C.fused_gemm_plan(bn, 1280, 8192, 0, 148, True, 0)
        assert bn_plan == bn
        per_cta = smem + r["smem"] + CTA_RESERVED_SMEM
        assert 2 * per_cta <= SM_SMEM, (r["kernel"], per_cta)
        # two accumulators of max(32, bn) columns each
        assert 2 * 2 * max(32, bn) <= TMEM_COLS
