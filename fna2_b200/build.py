"""Build ``libfna2_b200.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

Usage: ``python -m fna2_b200.build [--force] [--verbose]``.  The shared
library lands next to this file, so it travels with the source tree.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libfna2_b200.so")
SOURCES = ["fna2_api.cu"]
DEPS = ["fna2_api.cu", "fna2_fwd.cu", "fna2_gemm.cu", "fna2_bwd.cu", "fna2_noalloc.cu", "fna2_qkprep.cu", "fna2_decode.cu", "fna2_kernels.cuh", "ptx.cuh"]
HEADER = os.path.join(ROOT, "include", "fna2.h")


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def flags(verbose: bool = False):
    f = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
         "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    paths = [os.path.join(CSRC, d) for d in DEPS] + [HEADER]
    return any(os.path.getmtime(p) > t for p in paths)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + flags(verbose) + ["-o", tmp] + [os.path.join(CSRC, s) for s in SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libfna2_b200.so")
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
