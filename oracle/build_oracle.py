"""Builds the C oracle (oracle.c) into oracle/_build/liboracle.so with gcc + OpenMP.

TEST INFRASTRUCTURE: the library is the parity checker's fast twin and bench.py's timed
CPU baseline; the product never links it.  `-march=x86-64-v3` (AVX2/FMA) keeps the
binary portable to any current x86 server host of a B200 box.
"""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"


def build(force: bool = False) -> Path:
    src = HERE / "oracle.c"
    if not force and LIB.exists() and LIB.stat().st_mtime >= src.stat().st_mtime:
        return LIB
    LIB.parent.mkdir(parents=True, exist_ok=True)
    cc = shutil.which("gcc") or "cc"
    cmd = [cc, "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-o", str(LIB), str(src), "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
