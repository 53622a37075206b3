"""Builds libgaje_cuda.so in-tree for sm_100a (nvcc cross-compiles without a GPU).

The library is the product: the CUDA kernels, the host engine and the C ABI of
include/gaje_cuda.h.  The CUDA runtime is linked statically so the .so does not
depend on which libcudart the host process has already loaded.
"""
from __future__ import annotations

import os
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_PATH = os.path.join(PKG_DIR, "libgaje_cuda.so")
SOURCES = ["engine.cu", "flat_format.cpp"]
HEADERS = ["kernels.cuh", "megakernel.cuh", "fused.cuh", "gemm.cuh", "batch.cuh", "tc_gemm.cuh", "quant.cuh", "sample.cuh",
           "flat_format.h"]
NVCC = os.environ.get("GAJE_NVCC", "/usr/local/cuda/bin/nvcc")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    # every FMA in the kernels is an explicit fmaf(): no implicit contraction,
    # matching the Rust reference, which never contracts a*b+c
    "--fmad=false",
    "-ccbin", "/usr/bin/g++",
    "-Xcompiler", "-fPIC,-fopenmp,-ffp-contract=off,-O3",
    "-shared",
    "-cudart", "static",
]


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(REPO, "include", "gaje_cuda.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path."""
    if not force and not _stale():
        return LIB_PATH
    cmd = [NVCC, *NVCC_FLAGS, "-I", os.path.join(REPO, "include")]
    cmd += [os.path.join(CSRC, f) for f in SOURCES]
    cmd += ["-o", LIB_PATH + ".tmp", "-lgomp"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
