"""Build libmsattn.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

``python -m miniserve_b200.build`` or ``miniserve_b200.build.build()``.  The library lands in
``miniserve_b200/_lib/`` next to the sources so it travels with the source tree.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libmsattn.so"

SOURCES = [CSRC / "msattn.cu", CSRC / "plan.cpp", CSRC / "noalloc.cu"]
DEPS = [*SOURCES, *CSRC.glob("*.cuh"), ROOT / "include" / "msattn.h"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile (if stale) and return the library path."""
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc(),
        *ARCH,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-shared",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        "-I",
        str(ROOT / "include"),
        "-o",
        str(tmp),
        *map(str, SOURCES),
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
