"""Build recipe for the CPU oracle (test infrastructure, not product).

Compiles oracle/hxb_oracle.c with gcc + OpenMP into oracle/_lib/liboracle.so.
-ffp-contract=off keeps every multiply and add separately rounded, as the
linalg ops it restates are.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "hxb_oracle.c"
OUT_DIR = HERE / "_lib"
LIB = OUT_DIR / "liboracle.so"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= max(
            SRC.stat().st_mtime, Path(__file__).stat().st_mtime):
        return LIB
    OUT_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math",
           "-fopenmp", "-fPIC", "-shared", "-o", str(tmp), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
