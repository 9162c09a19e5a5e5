"""Compiler flags and sources of the native extension, shared by ``setup.py`` and
``comm_opt_b200.harness.ptxas_report`` (which compiles the same sources with ``-Xptxas -v``).

Loaded by file path (no package import), so it works before the extension exists.
"""
import os

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr"]
if os.environ.get("COB_CHECKED"):  # range-checked heap accesses in the collective kernels (debug builds)
    NVCC.append("-DCOB_CHECKED")
CXX = ["-O3", "-std=c++17"]

CUDA_SOURCES = ["fused_ar.cu", "fused_gemm.cu", "decode_ops.cu", "attention.cu", "gemm_sm100.cu", "probes.cu"]
SOURCES = ["bindings.cpp", "ops_bindings.cpp", "ipc_bindings.cpp", "tma_host.cpp"] + CUDA_SOURCES
