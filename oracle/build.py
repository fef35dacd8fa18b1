"""Build recipe for the CPU oracle (test infrastructure).

Compiles ``scalesweep_oracle.c`` with strict IEEE binary32 semantics into
``oracle/_build/libscalesweep_oracle.so``.  Nothing in the product links it.
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "scalesweep_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libscalesweep_oracle.so")

CFLAGS = ["-O2", "-fPIC", "-shared", "-fopenmp", "-fno-fast-math", "-ffp-contract=off",
          "-fno-builtin", "-std=c11", "-Wall", "-Wextra"]


def build(force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    if (not force and os.path.exists(LIB)
            and os.path.getmtime(LIB) >= os.path.getmtime(SRC)):
        return LIB
    tmp = LIB + ".tmp"
    subprocess.check_call(["gcc", *CFLAGS, SRC, "-o", tmp, "-lm"])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
