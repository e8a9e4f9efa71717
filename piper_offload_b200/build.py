"""Build ``libpiper_merge.so`` in-tree with nvcc for sm_100a.

Usage: ``python -m piper_offload_b200.build`` (also called by
``__graft_entry__.build()``). The build is skipped when the library is newer
than every source file.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
SOURCES = [PKG / "csrc" / "merge.cu"]
DEPS = SOURCES + [PKG / "csrc" / "ptx.cuh", PKG / "csrc" / "numerics.cuh", ROOT / "include" / "piper_merge.h"]
OUT = PKG / "libpiper_merge.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "--fmad=false",  # only the explicit fmaf() calls fuse, matching the reference's rounding points
    "-Xcompiler", "-fPIC",
    "-shared",
    # No --split-compile: its parallel device optimisation gave a different
    # binary on every build of the same source (instantiations measured up to
    # 20 % apart on a B200); one thread gives the same code each time.
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=str(ROOT))
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
