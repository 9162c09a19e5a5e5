"""Build of the comm_opt_b200 native extension (sm_100a only).

    python setup.py build_ext --inplace

produces comm_opt_b200/_C*.so next to the Python sources. Kernel sources (.cu) include no torch
headers; only the two binding files do, which keeps nvcc time low.
"""
import importlib.util
import os
from pathlib import Path

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "comm_opt_b200" / "csrc"

_spec = importlib.util.spec_from_file_location("cob_build_flags", CSRC / "build_flags.py")
flags = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(flags)

NVCC = flags.NVCC + ["-Xptxas=-v" if os.environ.get("COB_PTXAS_VERBOSE") else "-Xptxas=-O3"]
SOURCES = flags.SOURCES + [s for s in os.environ.get("COB_EXTRA_SOURCES", "").split(",") if s]

setup(
    name="comm_opt_b200",
    version="0.1.0",
    packages=["comm_opt_b200"],
    ext_modules=[
        CUDAExtension(
            name="comm_opt_b200._C",
            sources=[str(CSRC / s) for s in SOURCES],
            include_dirs=[str(CSRC)],
            extra_compile_args={"cxx": flags.CXX, "nvcc": NVCC},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
