"""Compile gate, after the reference's build check (scripts/build-local.sh:
77-130 requires every kernel to build with zero register spills): libgplk's
unity source compiles for sm_100a and ptxas reports no spill stores or
loads for any kernel. Runs on CPU (nvcc cross-compiles)."""
from __future__ import annotations

import re
import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
NVCC = "/usr/local/cuda/bin/nvcc"


@pytest.mark.skipif(not Path(NVCC).exists() and not shutil.which("nvcc"), reason="nvcc not available")
def test_every_kernel_builds_without_spills(tmp_path):
    nvcc = NVCC if Path(NVCC).exists() else shutil.which("nvcc")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
           "-shared", "-I", str(REPO / "include"), "-Xptxas", "-v", "-o", str(tmp_path / "libgplk_gate.so"),
           str(REPO / "gpu-power-lab_b200/csrc/gplk_unity.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    out = res.stdout + res.stderr
    kernels = re.findall(r"Function properties for (\S+)\n\s+(\d+) bytes stack frame, (\d+) bytes spill stores, "
                         r"(\d+) bytes spill loads", out)
    assert len(kernels) >= 20, "ptxas reported too few functions"
    spilling = [(name, st, ld) for name, _frame, st, ld in kernels if int(st) or int(ld)]
    assert not spilling, spilling
