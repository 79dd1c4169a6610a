"""Builds the CPU oracle (test infrastructure) as oracle/librec_oracle.so."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "rec_oracle.c"
LIB = HERE / "librec_oracle.so"
HEADER = HERE.parent / "include" / "rec_b200.h"

# IEEE single precision throughout: no contraction of a*b+c, FMA only where
# fmaf() is written; -mfma makes fmaf() a single instruction.
CFLAGS = ["-O2", "-mavx2", "-mfma", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared",
          "-fvisibility=hidden", "-Wall", "-Wno-unused-function", "-Wno-maybe-uninitialized"]


def build(verbose: bool = False) -> Path:
    if LIB.exists() and LIB.stat().st_mtime >= max(SRC.stat().st_mtime, HEADER.stat().st_mtime):
        return LIB
    cmd = ["gcc", *CFLAGS, str(SRC), "-o", str(LIB), "-lm"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
