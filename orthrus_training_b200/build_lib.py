"""Build liborthrus_b200.so (the C-ABI CUDA library) in-tree with nvcc for sm_100a.

    python -m orthrus_training_b200.build_lib [--force]

The whole library is one translation unit (csrc/capi.cu includes the kernel headers). The output
lands next to this file so it travels with the repository snapshot; it is rebuilt when a source is
newer than the library.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "liborthrus_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [
        ROOT / "include" / "orthrus_b200.h"]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    return any(p.stat().st_mtime > built for p in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    cmd = [NVCC, *FLAGS, f"-I{ROOT / 'include'}", f"-I{CSRC}", str(CSRC / "capi.cu"), "-o", str(LIB) + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    print("building", LIB.name, flush=True)
    subprocess.run(cmd, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
