"""Builds libw4a8.so (the C-ABI CUDA library) in-tree for sm_100a.

Usage: python build_native.py [--force]

The library is self-contained (static CUDA runtime, no torch linkage); the
Python module ``int4_int8_ext`` loads it with ctypes.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB = HERE / "libw4a8.so"
SOURCES = ["gemm_conv.cu", "aux_kernels.cu"]
HEADERS = ["ptx.cuh", "mma_kernel.cuh", "gemm_w4_kernel.cuh", "gemv_w4.cuh", "tensormap.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _stale() -> bool:
    if not LIB.exists():
        return True
    lib_t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [INCLUDE / "w4a8.h", Path(__file__)]
    return any(d.stat().st_mtime > lib_t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every CUDA source for sm_100a and links libw4a8.so."""
    if not force and not _stale():
        return LIB
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objs = []
    for src in SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp), *objs,
           "-Xcompiler", "-fPIC"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
