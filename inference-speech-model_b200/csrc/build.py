"""Builds libspd_b200.so (the C-ABI extension) for sm_100a with nvcc.

Usage:  python build.py [--verbose]   (from any directory)

Every ``*.cu`` file in this directory is compiled to an object with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` (in parallel), then linked
into ``../lib/libspd_b200.so`` with the CUDA runtime linked statically, so the library
carries no dependency on the CUDA runtime that the host process happens to load.
Objects are rebuilt only when a source or header is newer than them.

``python build.py --trace`` builds the trace variant instead: the same sources with
SPD_TRACE_BUILD defined, objects under ``_build/trace``, linked into
``../lib/libspd_b200_trace.so``.  Its kernels record a %globaltimer timeline of their
last launch (csrc/spd_trace.cuh); profile_cases.py at the repository root loads it with
``--trace``.  The normal library never contains these marks.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
REPO = PKG.parent
OBJ_DIR = PKG / "_build"
LIB = PKG / "lib" / "libspd_b200.so"
TRACE_OBJ_DIR = OBJ_DIR / "trace"
TRACE_LIB = PKG / "lib" / "libspd_b200_trace.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
                     "--expt-relaxed-constexpr", "-I", str(REPO / "include"), "-I", str(HERE)]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA extension cannot be built")
    return path


def _stale(obj: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False, trace: bool = False) -> Path:
    obj_dir, lib = (TRACE_OBJ_DIR, TRACE_LIB) if trace else (OBJ_DIR, LIB)
    flags = NVCC_FLAGS + (["-DSPD_TRACE_BUILD"] if trace else [])
    obj_dir.mkdir(parents=True, exist_ok=True)
    lib.parent.mkdir(parents=True, exist_ok=True)
    sources = sorted(HERE.glob("*.cu"))
    headers = sorted(HERE.glob("*.cuh")) + sorted((REPO / "include").glob("*.h"))
    cc = nvcc()
    jobs = []
    for src in sources:
        obj = obj_dir / (src.stem + ".o")
        if force or _stale(obj, [src] + headers):
            cmd = [cc] + flags + (["-Xptxas", "-v"] if verbose else []) + ["-c", str(src), "-o", str(obj)]
            jobs.append((src, cmd))
    def run(job):
        src, cmd = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r
    failed = []
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        for src, r in ex.map(run, jobs):
            if verbose or r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                failed.append(src.name)
    if failed:
        raise RuntimeError(f"nvcc failed for: {', '.join(failed)}")
    objs = [obj_dir / (s.stem + ".o") for s in sources]
    if force or jobs or not lib.exists() or _stale(lib, objs):
        cmd = [cc] + ARCH + ["-shared", "-cudart", "static", "-o", str(lib)] + [str(o) for o in objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError(f"linking {lib.name} failed")
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--trace", action="store_true", help="build the %%globaltimer trace variant")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force, trace=a.trace))
