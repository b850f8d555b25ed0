"""Build the sm_100a attention library in-tree: voxtral.cpp_b200/libvtx_fa.so.

    python voxtral.cpp_b200/build.py [--force] [--ptxas-verbose]

A plain nvcc invocation (no torch extension machinery): the product is a
C-ABI shared library that voxtral.cpp (or ctypes, cgo, ...) loads directly.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libvtx_fa.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def deps() -> list[str]:
    return sources() + sorted(glob.glob(os.path.join(HERE, "csrc", "*.cuh"))) + [
        os.path.join(ROOT, "include", "vtx_fa.h")]


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in deps())


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    if not force and not stale():
        return LIB
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
           "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared",
           "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp"]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    cmd += sources() + ["-lcudart"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.force or args.ptxas_verbose, args.ptxas_verbose))
    sys.exit(0)
