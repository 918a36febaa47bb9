"""Build libswiglu_b200.so in-tree with nvcc for sm_100a.

    python -m swiglu_b200.build [--force]      (run from swiglu-recompute_b200/)

The library is plain C ABI (include/swiglu_b200.h) linked against the static
CUDA runtime, so it needs no framework headers and loads on machines without a
GPU driver (CUDA is initialised lazily on the first call).
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
import tempfile

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)                      # swiglu-recompute_b200/
REPO_DIR = os.path.dirname(ROOT_DIR)
CSRC_DIR = os.path.join(ROOT_DIR, "csrc")
INCLUDE_DIR = os.path.join(REPO_DIR, "include")
LIB_NAME = "libswiglu_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libswiglu_b200.so")
    return cand


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC_DIR, "*.cu")))


def _inputs() -> list[str]:
    return (_sources() + sorted(glob.glob(os.path.join(CSRC_DIR, "*.cuh")))
            + sorted(glob.glob(os.path.join(INCLUDE_DIR, "*.h"))))


def is_stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    lib_m = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > lib_m for p in _inputs())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path."""
    if not force and not is_stale():
        return LIB_PATH
    fd, tmp = tempfile.mkstemp(suffix=".so", dir=PKG_DIR)
    os.close(fd)
    cmd = [_nvcc(), "-std=c++17", "-O3", *ARCH_FLAGS, "-lineinfo",
           "-Xcompiler", "-fPIC", "-shared", "-I", INCLUDE_DIR, "-I", CSRC_DIR,
           "-o", tmp, *_sources()]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    try:
        subprocess.run(cmd, check=True, stdout=None if verbose else subprocess.PIPE,
                       stderr=subprocess.STDOUT if not verbose else None)
    except subprocess.CalledProcessError as e:
        os.unlink(tmp)
        out = e.stdout.decode(errors="replace") if e.stdout else ""
        raise RuntimeError(f"nvcc failed:\n{out}") from None
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
