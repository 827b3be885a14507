"""Build recipe of the sm_100a extension (libtwilight_b200.so, in-tree).

    python twilight-cpu-gpu-offloading_b200/build.py

nvcc cross-compiles for sm_100a without a GPU.  The shared library exports
the C ABI declared in include/twilight_b200.h.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libtwilight_b200.so"
SOURCES = ["quest.cu", "int4.cu", "topp_union.cu", "gather.cu", "attention.cu", "frontend.cu",
           "capi.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the sm_100a extension cannot be built")


def sources() -> list[Path]:
    return [CSRC / s for s in SOURCES]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + [REPO / "include" / "twilight_b200.h"]
    return any(d.stat().st_mtime > mtime for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, *map(str, sources()), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
