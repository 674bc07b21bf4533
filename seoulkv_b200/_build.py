"""Build the in-tree CUDA library (sm_100a) with nvcc.

``python seoulkv_b200/_build.py [--force] [-v]`` (or ``__graft_entry__.build()``) compiles
``csrc/*.cu`` into ``seoulkv_b200/_lib/libseoulkv_b200.so``.  The library is
built in the source tree so it travels with the repository to a GPU host.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libseoulkv_b200.so"
SOURCES = ("skv_kernels.cu", "skv_fused.cu", "skv_shard.cu", "skv_append.cu", "skv_engine.cu", "skv_noalloc.cu")
ARCH = ("-gencode", "arch=compute_100a,code=sm_100a")


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def stale() -> bool:
    if not LIB.exists():
        return True
    newest = max(p.stat().st_mtime for p in list(CSRC.glob("*.cu*")) + [PKG.parent / "include" / "seoulkv_b200.h"])
    return LIB.stat().st_mtime < newest


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-o", str(tmp), *(str(CSRC / s) for s in SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
