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
from concurrent.futures import ThreadPoolExecutor
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
    """Compiles every source to an object in parallel (one nvcc per file),
    then links the shared library."""
    if not force and not needs_build():
        return LIB
    obj_dir = PKG / "_build"
    obj_dir.mkdir(exist_ok=True)
    compile_flags = [f for f in NVCC_FLAGS if f != "-shared"]
    jobs = []
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        jobs.append((obj, [nvcc(), *compile_flags, "-c", str(src), "-o", str(obj)]))
    if verbose:
        for _, cmd in jobs:
            print(" ".join(cmd))
    workers = max(1, min(len(jobs), os.cpu_count() or 1))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        results = list(pool.map(lambda j: subprocess.run(j[1]).returncode, jobs))
    if any(results):
        raise RuntimeError(f"nvcc failed for {[str(j[0].name) for j, r in zip(jobs, results) if r]}")
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
            *[str(o) for o, _ in jobs], "-o", str(tmp)]
    if verbose:
        print(" ".join(link))
    subprocess.run(link, check=True)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
