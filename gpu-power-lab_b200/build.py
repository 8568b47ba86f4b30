"""Build libgplk.so (the sm_100a kernel library and its C ABI) in-tree.

    python gpu-power-lab_b200/build.py [--verbose]

nvcc cross-compiles for sm_100a without a GPU. The library is one
translation unit (csrc/gplk_unity.cu) linked with the static CUDA runtime,
so it does not depend on which libcudart another library in the process
brought along.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libgplk.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-I", str(REPO / "include"),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise FileNotFoundError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted((REPO / "include").glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources())


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *NVCC_FLAGS]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    tmp = LIB.with_suffix(".so.tmp")
    cmd += ["-o", str(tmp), str(CSRC / "gplk_unity.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libgplk.so")
    if verbose:
        sys.stderr.write(res.stderr)
    tmp.replace(LIB)
    return LIB


NODEMON = PKG / "libgplk_nodemon.so"


def build_nodemon(force: bool = False) -> Path:
    """libgplk_nodemon.so: the node-level NVML sampler (host C, no CUDA code;
    NVML is loaded at run time with dlopen)."""
    src = CSRC / "gplk_nodemon.c"
    hdr = REPO / "include" / "gplk_nodemon.h"
    if not force and NODEMON.exists() and NODEMON.stat().st_mtime >= max(src.stat().st_mtime, hdr.stat().st_mtime):
        return NODEMON
    cmd = ["gcc", "-std=gnu11", "-O2", "-Wall", "-fPIC", "-shared", "-I", "/usr/local/cuda/include",
           "-o", str(NODEMON), str(src), "-ldl", "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("gcc failed building libgplk_nodemon.so")
    return NODEMON


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force=True)
    build_nodemon(force=True)
    print(LIB)
    print(NODEMON)
