"""The node-level power sampler (libgplk_nodemon.so) on CPU, against a fake
NVML (tests/csrc/fake_nvml.c: a square wave on the host clock, a driver
sample every 20 ms). Checks the polled and buffered paths, the shared
timebase, the node-level sum, and aligned versus staggered phase."""
from __future__ import annotations

import os
import subprocess
import time
from pathlib import Path

import numpy as np
import pytest

from gplk import nodemon

REPO = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def fake_nvml(tmp_path_factory):
    out = tmp_path_factory.mktemp("nvml") / "libfake_nvml.so"
    subprocess.run(["gcc", "-std=gnu11", "-O2", "-fPIC", "-shared", "-I/usr/local/cuda/include", "-o", str(out),
                    str(REPO / "tests/csrc/fake_nvml.c")], check=True)
    if not nodemon.LIB_PATH.exists():
        import importlib.util

        spec = importlib.util.spec_from_file_location("gplk_build", REPO / "gpu-power-lab_b200" / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build_nodemon(force=True)
    return str(out)


def _run(fake, devices, seconds, hz=200, drain_ms=50, stagger=False):
    os.environ["FAKE_NVML_STAGGER"] = "1" if stagger else "0"
    os.environ["FAKE_NVML_NDEV"] = str(len(devices))
    mon = nodemon.NodeMonitor(devices, hz=hz, drain_ms=drain_ms, nvml_path=fake)
    time.sleep(seconds)
    mon.stop()
    return mon


def test_polled_and_buffered_paths(fake_nvml):
    mon = _run(fake_nvml, [0, 1], 0.8)
    try:
        s = mon.samples()
        for dev in (0, 1):
            p = s[(s["device"] == dev) & (s["source"] == nodemon.POLLED)]
            b = s[(s["device"] == dev) & (s["source"] == nodemon.BUFFERED)]
            assert 0.6 * 200 * 0.8 <= len(p) <= 1.2 * 200 * 0.8, len(p)
            assert np.all(np.diff(p["t_s"]) > 0)
            assert set(np.unique(p["power_w"])) <= {300.0, 900.0}
            assert np.allclose(p["instant_w"] - p["power_w"], 50.0, atol=0.01) or (
                np.mean(np.abs(p["instant_w"] - p["power_w"] - 50.0) < 0.01) > 0.95)  # a read may straddle an edge
            # the driver buffer: one sample per 20 ms, strictly increasing, none before the monitor started
            assert len(b) >= 0.8 / 0.02 * 0.8
            assert np.all(np.diff(b["t_s"]) > 0) and np.allclose(np.diff(b["t_s"]), 0.02, atol=1e-6)
            assert b["t_s"][0] > -0.021 and np.all(b["instant_w"] == -1.0)
    finally:
        mon.close()


def test_node_sum_aligned_vs_staggered(fake_nvml):
    results = {}
    for stagger in (False, True):
        mon = _run(fake_nvml, [0, 1, 2, 3], 1.0, stagger=stagger)
        try:
            w = mon.node_series(nodemon.BUFFERED, t0=0.0, bin_s=0.02, max_bins=1000)
            w = w[5:-2]  # every device has started
            results[stagger] = (np.percentile(w, 95) - np.percentile(w, 5), float(np.mean(w)))
        finally:
            mon.close()
    swing_aligned, mean_aligned = results[False]
    swing_staggered, mean_staggered = results[True]
    assert swing_aligned == pytest.approx(4 * 600.0, abs=1.0)   # all four swing together
    assert swing_staggered <= 600.0 + 1.0                       # at most one edge in flight
    assert mean_aligned == pytest.approx(4 * 600.0, rel=0.1)    # same energy either way
    assert mean_staggered == pytest.approx(4 * 600.0, rel=0.1)


def test_bad_arguments(fake_nvml, tmp_path):
    with pytest.raises(nodemon.NodeMonitorError):
        nodemon.NodeMonitor([0], hz=0, nvml_path=fake_nvml)
    with pytest.raises(nodemon.NodeMonitorError):
        nodemon.NodeMonitor([0], nvml_path=str(tmp_path / "missing.so"))
    with pytest.raises(nodemon.NodeMonitorError):
        nodemon.NodeMonitor([9], nvml_path=fake_nvml)  # no such device
