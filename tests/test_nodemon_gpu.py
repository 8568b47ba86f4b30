"""The node-level power sampler (libgplk_nodemon.so) on the GPU box's real
NVML, around a 300 ms triad burst: both the polled path and the driver's
buffered samples (nvmlDeviceGetSamples, the path the reference's probe
checks at runner/src/probe.c:58-65) return samples, their timestamps are
monotonic per device and source, and the burst draws more power than the
idle floor before it. The sampler only reads NVML."""
from __future__ import annotations

import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_real_nvml_polled_and_buffered_during_burst(gplk, cuda):
    import torch

    from gplk import nodemon

    n = 1 << 28  # 3 x 1 GiB: each triad ~0.5 ms, so a 300 ms burst is ~600 launches
    b = torch.rand(n, device=cuda)
    c = torch.rand(n, device=cuda)
    a = torch.empty(n, device=cuda)
    torch.cuda.synchronize()
    t_open = time.time()  # sample times count from the monitor's opening
    mon = nodemon.NodeMonitor([cuda.index or 0], hz=100, drain_ms=50)
    try:
        time.sleep(0.4)  # idle floor
        t_burst = time.time()
        while time.time() - t_burst < 0.3:
            for _ in range(32):
                gplk.triad(a, b, c, 3.0)
            torch.cuda.synchronize()
        t_end = time.time()
        t_burst, t_end = t_burst - t_open, t_end - t_open
        time.sleep(0.3)
        mon.stop()
        s = mon.samples()
    finally:
        mon.close()
    polled = s[s["source"] == nodemon.POLLED]
    buffered = s[s["source"] == nodemon.BUFFERED]
    assert len(polled) >= 50, len(polled)
    assert len(buffered) >= 5, len(buffered)
    for part in (polled, buffered):
        assert np.all(np.diff(part["t_s"]) >= 0.0)
        assert np.all(part["power_w"] > 0.0)
    # The burst window's power against the idle window before it, on the
    # polled path (driver-averaged, so it lags: compare the burst's maximum).
    idle = polled[polled["t_s"] < t_burst - 0.05]["power_w"]
    burst = polled[(polled["t_s"] >= t_burst) & (polled["t_s"] <= t_end + 0.2)]["power_w"]
    assert len(idle) > 5 and len(burst) > 5
    assert float(burst.max()) > float(np.median(idle)) + 20.0, (float(np.median(idle)), float(burst.max()))
