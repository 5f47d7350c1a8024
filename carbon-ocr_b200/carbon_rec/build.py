"""Builds the CUDA library in-tree: csrc/*.cu -> carbon_rec/libcarbon_rec.so for sm_100a.

nvcc cross-compiles without a GPU, so this runs on any machine with the CUDA toolkit.
Host code is compiled without floating-point contraction (the crop rule's double
arithmetic must round as the reference's does); device code with -fmad=false for the
same reason, the kernels spelling out every fused multiply-add they want.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parent.parent / "include"
LIB = PKG / "libcarbon_rec.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "carbon_rec.h"]


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++20", "-fmad=false", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden", "-shared",
           f"-I{INCLUDE}", str(CSRC / "crec.cu"), "-o", str(LIB)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libcarbon_rec.so")
    if verbose:
        sys.stderr.write(r.stderr)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
