"""Build recipe of the CPU oracle (test infrastructure only).

Compiles ``oracle/oracle.cpp`` and ``oracle/dejavu.cpp`` into ``oracle/liboracle.so`` with the flags the
parity argument depends on: ``-ffp-contract=off`` (the Rust reference never
fuses a*b+c) and no fast-math.  ``-march=x86-64-v3`` (AVX2/FMA level) keeps the
library loadable on the GPU box's host CPU.  OpenMP drives the HOGWILD
baseline.

The Rust reference itself cannot be compiled here (no cargo/rustc, no crate
registry), so there is no ``oracle/_ref`` build.
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "oracle.cpp"
SRCS = [SRC, HERE / "dejavu.cpp"]
LIB = HERE / "liboracle.so"
HDR = HERE.parent / "include" / "klearu_gpu.h"
FLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math", "-fopenmp",
         "-fPIC", "-shared", "-std=c++17"]


def build_oracle(force: bool = False) -> Path:
    newest = max(max(p.stat().st_mtime for p in SRCS), HDR.stat().st_mtime)
    if not force and LIB.exists() and LIB.stat().st_mtime > newest:
        return LIB
    cmd = ["g++", *FLAGS, *map(str, SRCS), "-o", str(LIB)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("oracle build failed")
    return LIB


if __name__ == "__main__":
    print(build_oracle(force="-f" in sys.argv))
