"""Build libqwz_b200.so (sm_100a) in-tree with nvcc.

The library is one translation unit (csrc/qwz_b200.cu) compiled for
``-gencode arch=compute_100a,code=sm_100a``; the static CUDA runtime is linked
in, so the .so only needs the driver at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libqwz_b200.so"
SOURCES = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [
    PKG.parent / "include" / "qwz_b200.h"
]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libqwz_b200.so")


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    mtime = LIB.stat().st_mtime
    return all(src.stat().st_mtime <= mtime for src in SOURCES if src.exists())


def build(force: bool = False, verbose: bool = False, ptxas_report: bool = False) -> Path:
    """Compile the library unless it is newer than every source."""
    if not force and up_to_date():
        return LIB
    cmd = [nvcc_path(), *NVCC_FLAGS]
    if ptxas_report:
        cmd += ["-Xptxas", "-v"]
    tmp = LIB.with_suffix(".so.tmp")
    cmd += [str(CSRC / "qwz_b200.cu"), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    proc = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stderr}")
    if verbose or ptxas_report:
        print(proc.stderr, file=sys.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_report="-v" in sys.argv)
    print(LIB)
