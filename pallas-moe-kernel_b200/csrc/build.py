"""Builds ``libmoe_b200.so`` (sm_100a) from the CUDA sources in this folder.

Output: ``<package>/lib/libmoe_b200.so``.  nvcc cross-compiles for sm_100a
without a GPU.  The build is skipped when the library is newer than every
source and header.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
REPO = PKG.parent
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libmoe_b200.so"
SOURCES = ["moe_b200.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _deps() -> list[Path]:
    files = [p for p in CSRC.iterdir() if p.suffix in (".cu", ".cuh", ".h")]
    files += list((REPO / "include").glob("*.h"))
    return files


def build(force: bool = False, verbose: bool = False) -> Path:
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    if LIB.exists() and not force:
        lib_t = LIB.stat().st_mtime
        if all(p.stat().st_mtime <= lib_t for p in _deps()):
            return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "-shared",
           "-I", str(REPO / "include"), "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True, cwd=str(CSRC))
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    out = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(out)
