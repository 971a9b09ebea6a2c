"""Builds the CPU oracle (test infrastructure only): oracle/_build/liboracle.so.

    python -m oracle.build

gcc -O2 -fopenmp -ffp-contract=off: no step is fused into an fma unless the source calls
fmaf, so the deterministic sigmoid and the RoPE table reproduce bit for bit.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "hk_oracle.c"
OUT = HERE / "_build"
LIB = OUT / "liboracle.so"


def build(force: bool = False) -> Path:
    OUT.mkdir(exist_ok=True)
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-std=c11",
           str(SRC), "-o", str(LIB), "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed: {' '.join(cmd)}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
