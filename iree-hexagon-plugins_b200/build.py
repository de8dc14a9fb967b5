"""Build recipe for libhxb200.so, the sm_100a dispatch library.

Compiles every csrc/*.cu with nvcc for sm_100a only (no PTX fallback, no other
architectures), links the CUDA runtime statically and writes the shared library
next to this file, so that it travels with the source tree. Usage:

    python iree-hexagon-plugins_b200/build.py [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "libhxb200.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-I", str(PKG_DIR.parent / "include"),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the dispatch library needs the CUDA toolkit")


CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-I", str(PKG_DIR.parent / "include")]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _host_sources() -> list[Path]:
    """Host-only C++ (the compiler stand-in), built with the host compiler."""
    return sorted((CSRC / "compiler").glob("*.cc"))


def _deps() -> list[Path]:
    return sorted([p for p in CSRC.rglob("*") if p.is_file()] +
                  list((PKG_DIR.parent / "include").glob("*.h")))


def _needs_build(force: bool) -> bool:
    if force or not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > lib_mtime for p in _deps() + [Path(__file__)])


def _compile(nvcc: str, src: Path, extra: list[str]) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def _compile_host(src: Path) -> Path:
    obj = BUILD_DIR / (src.stem + ".host.o")
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    cmd = [cxx, *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{cxx} failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, extra: list[str] | None = None) -> Path:
    """Builds libhxb200.so if any source is newer than it; returns its path."""
    if not _needs_build(force):
        return LIB_PATH
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    extra = list(extra or [])
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, extra), srcs))
        objs += list(ex.map(_compile_host, _host_sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
           "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_verbose else []
    print(build(force=a.force or a.ptxas_verbose, jobs=a.jobs, extra=extra))
    sys.exit(0)
