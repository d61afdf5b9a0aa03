"""Build the CPU oracle shared library (test infrastructure only).

    python oracle/build.py

Compiles sv_oracle.c into oracle/liboracle_sv.so with gcc.  -ffp-contract=off keeps
the compiler from fusing multiply-adds the source does not spell out as fmaf/fma,
so the oracle's float arithmetic is exactly what the source says.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "sv_oracle.c")
LIB = os.path.join(HERE, "liboracle_sv.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp",
           "-shared", "-fPIC", "-o", LIB, SRC, "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
