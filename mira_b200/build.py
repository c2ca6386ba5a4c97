"""Builds libmira_cuda.so in-tree with nvcc for sm_100a (no CUDA device needed)."""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libmira_cuda.so"
INCLUDE = PKG.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
    # no --use_fast_math: the epilogue relies on IEEE division/rounding and explicit intrinsics
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libmira_cuda.so")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "mira_cuda.h"]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(s.stat().st_mtime <= t for s in sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> Path:
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, *(extra or []), "-I", str(INCLUDE), str(CSRC / "mira_cuda.cu"), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    args = sys.argv[1:]
    out = build(force="--force" in args, verbose=True, extra=[a for a in args if a.startswith("-X") and a != "--force"])
    print(out)
