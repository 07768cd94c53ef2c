"""Builds the in-tree CUDA library (sm_100a) from mac-ai-engineering_b200/csrc:

    python -m macai_b200.build          (from mac-ai-engineering_b200/)

nvcc compiles every .cu into one shared object, libgated_delta_b200.so, next to this file. The C ABI it exports is
include/gated_delta_b200.h at the repository root. nvcc cross-compiles: no GPU is needed to build.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
SRC_ROOT = os.path.dirname(PKG)                       # mac-ai-engineering_b200/
REPO = os.path.dirname(SRC_ROOT)
CSRC = os.path.join(SRC_ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_NAME = "libgated_delta_b200.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-shared"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit (12.8+) is needed to build the sm_100a library")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    newest = max(os.path.getmtime(p) for p in sources() + glob.glob(os.path.join(CSRC, "*.cuh")) +
                 glob.glob(os.path.join(INCLUDE, "*.h")))
    return os.path.getmtime(LIB_PATH) >= newest


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if a source is newer than it (or force). Returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", INCLUDE, "-I", CSRC, "-o", tmp, *sources()]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
