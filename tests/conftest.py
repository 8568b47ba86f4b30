"""Shared pytest setup: the `gpu` marker, import paths, and fixtures.

`-m "not gpu"` runs the oracle, host logic and C-ABI export checks on any
machine; `-m gpu` runs the parity tests against the oracle on a B200.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "gpu-power-lab_b200"
for p in (PKG, REPO / "oracle", REPO):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def reference_root() -> Path | None:
    """The gpu-power-lab source tree the parity recipes were built from:
    $GPL_REFERENCE_ROOT, else the path oracle/ref_build.sh recorded in
    oracle/_ref/reference_root. None when neither names an existing tree
    (the tests that read the reference's schema or host sources then skip)."""
    import os

    cand = os.environ.get("GPL_REFERENCE_ROOT")
    rec = REPO / "oracle" / "_ref" / "reference_root"
    if not cand and rec.exists():
        cand = rec.read_text().strip()
    if cand and Path(cand).is_dir():
        return Path(cand)
    return None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o

    o.lib()
    return o


@pytest.fixture(scope="session")
def gplk():
    import gplk as g

    g.lib()
    return g


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA (run with -m 'not gpu')")
    torch.cuda.init()
    return torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """Every GPU test must leave the library's device status word at OK."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import gplk as g

    code, site = g.status_read(clear=True)
    assert code == 0, f"device status {g.STATUS.get(code, code)} at site {site:#x}"
