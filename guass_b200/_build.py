"""Build libgfield.so in-tree with nvcc for sm_100a.

The library is plain CUDA C++ behind a C ABI (include/gfield.h); it is built
with explicit nvcc flags (no torch extension machinery) so the same .so can be
loaded from Python (ctypes), C, or any FFI.  It must be built without
--use_fast_math: the renderer relies on CUDA's IEEE expf/log1pf/div/sqrt to
match the reference bit for bit.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
SOURCES = [PKG / "csrc" / "gfield.cu"]
HEADERS = [ROOT / "include" / "gfield.h"]
LIB = PKG / "libgfield.so"
# debug build: every shape-derived global access bounds-checked (GF_FLAG_BOUNDS);
# load it instead of the release library with GUASS_B200_LIB=<path>
LIB_CHECK = PKG / "libgfield_check.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def needs_build(lib: Path = LIB) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False, check: bool = False) -> Path:
    """Build the release library (or, with ``check``, the bounds-checked one)."""
    lib = LIB_CHECK if check else LIB
    if not force and not needs_build(lib):
        return lib
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, *(["-DGF_CHECK"] if check else []), f"-I{ROOT / 'include'}", *map(str, SOURCES),
           "-o", str(tmp), "-lcudart"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, lib)
    return lib


def build_all(force: bool = False, verbose: bool = False) -> list[Path]:
    return [build(force, verbose), build(force, verbose, check=True)]


if __name__ == "__main__":
    for lib in build_all(force="--force" in sys.argv, verbose=True):
        print(lib)
