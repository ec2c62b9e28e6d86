"""Build the native sm_100a extension in place: ``python setup.py build_ext --inplace``.

Produces ``packbalance_b200/_C*.so``.  Only ``sm_100a`` code is generated; the build
runs on machines without a GPU (nvcc cross-compiles).
"""

import os
from pathlib import Path

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

os.environ["TORCH_CUDA_ARCH_LIST"] = ""  # the explicit -gencode below is the only target
os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))

ROOT = Path(__file__).parent
CSRC = ROOT / "packbalance_b200" / "csrc"
SOURCES = ["bindings.cpp", "gemm.cu", "elementwise.cu", "attention.cu", "comm.cu", "fsdp.cu", "noalloc.cu"]
SOURCES = [str((CSRC / s).relative_to(ROOT)) for s in SOURCES]
# PB_DEBUG_BOUNDS=1 builds the index checks of csrc/common.cuh (PB_BOUNDS_OK) into the
# kernels: a bad work item, owner rank or token id is reported through the device status
# word and its access skipped.  Rebuild without it for normal use.
DEFINES: list[str] = ["-DPB_DEBUG_BOUNDS"] if os.environ.get("PB_DEBUG_BOUNDS") == "1" else []

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("PB_PTXAS_VERBOSE") else "-Xptxas=-O3",
    *DEFINES,
]

setup(
    name="packbalance_b200",
    version="0.1.0",
    packages=find_packages(include=["packbalance_b200*"]),
    ext_modules=[
        CUDAExtension(
            name="packbalance_b200._C",
            sources=SOURCES,
            extra_compile_args={"cxx": ["-O3", "-std=c++17", *DEFINES], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
