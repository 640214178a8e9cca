"""Builds libdiffrast_cuda.so in-tree with nvcc for sm_100a (B200).

    python differentiable-rasterizer_b200/build_native.py [--force]

The library is the C ABI of include/diffrast_cuda.h. The CUDA runtime is linked
statically, so the .so depends only on the driver and runs in any process,
with or without torch. Output: differentiable-rasterizer_b200/diffrast/libdiffrast_cuda.so
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
SOURCES = [os.path.join(CSRC, f) for f in ("dr_kernels.cu", "dr_capi.cu", "dr_noalloc.cu")]
HEADERS = [
    os.path.join(CSRC, "dr_device.cuh"),
    os.path.join(CSRC, "dr_internal.h"),
    os.path.join(CSRC, "dr_math.cuh"),
    os.path.join(REPO, "include", "diffrast_cuda.h"),
]
LIB = os.path.join(HERE, "diffrast", "libdiffrast_cuda.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libdiffrast_cuda.so")


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in SOURCES + HEADERS + [__file__])


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *NVCC_FLAGS, "-shared", "-o", tmp, *SOURCES,
           "-Xlinker", "--exclude-libs,ALL"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
