"""Build libssparse.so in-tree for sm_100a (nvcc, one shared library, no torch extension).

    python -m streaming_sparse_b200.build            # incremental
    python -m streaming_sparse_b200.build --force    # rebuild
    python -m streaming_sparse_b200.build --verbose  # also print ptxas register/smem usage
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libssparse.so")
ROOT = os.path.dirname(PKG)
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
         "-I", os.path.join(ROOT, "include")]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(ROOT, "include", "ssparse.h")]
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not verbose and not _stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [NVCC, *ARCH, *FLAGS, *(["-Xptxas", "-v"] if verbose else []), "-o", tmp, *sources()]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libssparse.so")
    if verbose:
        sys.stderr.write(r.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
