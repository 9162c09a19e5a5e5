"""Build of the comm_opt_b200 native extension (sm_100a only).

    python setup.py build_ext --inplace

produces comm_opt_b200/_C*.so next to the Python sources. Kernel sources (.cu) include no torch
headers; only the two binding files do, which keeps nvcc time low.
"""
import os
from pathlib import Path

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "comm_opt_b200" / "csrc"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xptxas=-v" if os.environ.get(
    "COB_PTXAS_VERBOSE") else "-Xptxas=-O3"]
if os.environ.get("COB_CHECKED"):  # range-checked heap accesses in the collective kernels (debug builds)
    NVCC.append("-DCOB_CHECKED")
CXX = ["-O3", "-std=c++17"]

SOURCES = [
    "bindings.cpp",
    "ops_bindings.cpp",
    "ipc_bindings.cpp",
    "fused_ar.cu",
    "fused_gemm.cu",
    "decode_ops.cu",
    "attention.cu",
    "gemm_sm100.cu",
    "tma_host.cpp",
    "probes.cu",
]
SOURCES += [s for s in os.environ.get("COB_EXTRA_SOURCES", "").split(",") if s]

setup(
    name="comm_opt_b200",
    version="0.1.0",
    packages=["comm_opt_b200"],
    ext_modules=[
        CUDAExtension(
            name="comm_opt_b200._C",
            sources=[str(CSRC / s) for s in SOURCES],
            include_dirs=[str(CSRC)],
            extra_compile_args={"cxx": CXX, "nvcc": NVCC},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
