"""Build recipe for libctfa_b200.so (sm_100a only).

``python -m cudatransformer_b200.build`` compiles csrc/ctfa_api.cu with nvcc
into the package directory, where ``_lib.load()`` picks it up.  nvcc
cross-compiles without a GPU.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
SRC = PKG / "csrc" / "ctfa_api.cu"
OUT = PKG / "libctfa_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def sources() -> list[Path]:
    return sorted((PKG / "csrc").glob("*.cu*")) + [PKG.parent / "include" / "ctfa.h"]


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    cmd = [NVCC, *FLAGS, str(SRC), "-o", str(OUT)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
