"""Build the sm_100a CUDA library ``libscalesweep_b200.so`` in-tree.

    python -m test_speed_scalesweep_b200.build [--force]

nvcc cross-compiles for ``-gencode arch=compute_100a,code=sm_100a`` without a
GPU.  The library links the CUDA runtime dynamically (``-cudart shared``), so
inside a PyTorch process it shares torch's already-loaded libcudart.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB_NAME = "libscalesweep_b200.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)
BUILD_DIR = os.path.join(PKG, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return (sources() + glob.glob(os.path.join(CSRC, "*.cuh")) +
            glob.glob(os.path.join(INCLUDE, "*.h")))


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(d) <= t for d in _deps())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(BUILD_DIR, exist_ok=True)
    nvcc = _nvcc()
    objs = []
    for src in sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj]
        if verbose:
            cmd += ["-Xptxas", "-v"]
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        objs.append(obj)
    tmp = LIB_PATH + ".tmp"
    cuda_lib = os.path.join(os.path.dirname(os.path.dirname(os.path.realpath(nvcc))), "lib64")
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "shared", "-o", tmp, *objs,
           "-Xlinker", "-rpath=" + cuda_lib]
    subprocess.check_call(cmd)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
