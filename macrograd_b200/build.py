"""Builds the in-tree shared library macrograd_b200/libmg_gemm.so for sm_100a.

    python -m macrograd_b200.build        (or build() from Python)

nvcc cross-compiles without a GPU. The library links the CUDA runtime
statically and reaches the driver's tensor-map encoder through
cudaGetDriverEntryPoint, so it needs no libcuda at link time.
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "libmg_gemm.so")
SOURCES = [os.path.join(PKG, "csrc", "mg_gemm.cu")]
DEPS = SOURCES + [
    os.path.join(PKG, "csrc", "mg_gemm_kernel.cuh"),
    os.path.join(PKG, "csrc", "mg_ptx.cuh"),
    os.path.join(ROOT, "include", "mg_gemm.h"),
]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(home, "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in DEPS if os.path.exists(p))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-I" + os.path.join(ROOT, "include"), "-o", LIB, *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
