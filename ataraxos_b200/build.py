"""Build libstratego_b200.so for sm_100a (``python -m ataraxos_b200.build``).

The library is compiled in-tree with nvcc into ``ataraxos_b200/_lib/`` so it
travels with the source tree; nothing is JIT-compiled at import time.
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
INCLUDE = ROOT / "include"
LIB_DIR = PKG / "_lib"
LIB_PATH = LIB_DIR / "libstratego_b200.so"
# the debug build: every kernel checks each game record's indices first (SB_DEBUG_BOUNDS)
DEBUG_LIB_PATH = LIB_DIR / "libstratego_b200_debug.so"
SOURCES = [CSRC / "sb_kernels.cu"]
DEPS = SOURCES + [CSRC / "sb_device.cuh", INCLUDE / "stratego_b200.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-shared", "-Xcompiler", "-fPIC",
]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise FileNotFoundError("nvcc not found: the CUDA toolkit is needed to build libstratego_b200.so")


def up_to_date(path: Path = LIB_PATH) -> bool:
    if not path.exists():
        return False
    t = path.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in DEPS)


def _compile(path: Path, extra: list[str], verbose: bool) -> None:
    LIB_DIR.mkdir(exist_ok=True)
    tmp = path.with_name(f".{path.name}.{os.getpid()}.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, *extra, f"-I{INCLUDE}", "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, path)


def build(force: bool = False, verbose: bool = False, debug: bool = True) -> Path:
    """Build the production library (and, with ``debug``, the bounds-checking one)."""
    if force or not up_to_date(LIB_PATH):
        _compile(LIB_PATH, [], verbose)
    if debug and (force or not up_to_date(DEBUG_LIB_PATH)):
        _compile(DEBUG_LIB_PATH, ["-DSB_DEBUG_BOUNDS"], verbose)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
