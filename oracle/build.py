"""Build recipe of the CPU oracle (test infrastructure): compiles
oracle/tb_oracle.cpp into oracle/libtb_oracle.so with g++ (OpenMP, no
fast-math, no FP contraction, portable x86-64-v3 code so the library built
here also runs on the GPU host).

    python oracle/build.py [--force]
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "tb_oracle.cpp"
HDR = HERE / "tb_oracle.h"
LIB = HERE / "libtb_oracle.so"
FLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
         "-fPIC", "-shared", "-std=c++17"]


def build(force: bool = False) -> Path:
    if (not force and LIB.exists()
            and LIB.stat().st_mtime >= max(SRC.stat().st_mtime, HDR.stat().st_mtime)):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = ["g++"] + FLAGS + [str(SRC), "-o", str(tmp)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
