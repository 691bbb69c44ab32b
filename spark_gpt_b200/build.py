"""Build libb200moe.so in-tree with nvcc for sm_100a.

    python -m spark_gpt_b200.build [--force]

The library is a plain C-ABI shared object (include/b200moe.h); it links only
against the CUDA runtime, so no torch headers are involved.
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
LIB = PKG / "libb200moe.so"
SOURCES = [CSRC / "b200moe.cu"]
DEPS = SOURCES + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "b200moe.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
    "-cudart", "static",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the B200 MoE library needs the CUDA toolkit to build")
    return cand


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-o", str(tmp),
           *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
