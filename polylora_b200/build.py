"""Builds libpolylora_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

Usage: ``python -m polylora_b200.build`` (or ``build()`` from Python).  The
shared object lands next to this file in ``_lib/`` so that it travels with the
source tree; it links the CUDA runtime statically and needs only the driver
at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libpolylora_b200.so"
INCLUDE_DIR = PKG_DIR.parent / "include"

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O2",
    "-shared",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE_DIR / "polylora_b200.h"]


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    mtime = LIB_PATH.stat().st_mtime
    return all(src.stat().st_mtime <= mtime for src in _sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles the library unless it is newer than every source file."""
    if not force and up_to_date():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", str(INCLUDE_DIR), "-o", str(tmp), str(CSRC / "plora.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
