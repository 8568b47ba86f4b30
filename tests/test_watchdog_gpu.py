"""Failure detection without a GPU fault: every device wait in libgplk is
bounded. A wait that can never complete gives up after its budget, the
library's status word reports the timeout and where, and the context keeps
working."""
from __future__ import annotations

import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports(gplk, oracle, cuda):
    import torch

    gplk.status_read(clear=True)
    gave_up = torch.zeros(1, dtype=torch.int32, device=cuda)
    t0 = time.perf_counter()
    gplk.selftest_wait_timeout(50_000_000, gave_up)  # 50 ms budget
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(gave_up.item()) == 1
    assert 0.04 <= elapsed < 5.0, elapsed
    code, site = gplk.status_read(clear=True)
    assert code == 3 and site == 0x0F01, (code, hex(site))
    # the context is intact: a triad still runs bit-exact afterwards
    n = 4099
    b = oracle.uniform_f32(n, 1)
    c = oracle.uniform_f32(n, 2)
    a = torch.empty(n, device=cuda)
    gplk.triad(a, torch.from_numpy(b).to(cuda), torch.from_numpy(c).to(cuda), 3.0)
    torch.cuda.synchronize()
    assert np.array_equal(a.cpu().numpy().view(np.uint32), oracle.triad_f32(b, c, 3.0).view(np.uint32))


def test_selftest_rejects_unbounded_budget(gplk, cuda):
    with pytest.raises(gplk.GplkError):
        gplk.selftest_wait_timeout(0)
    with pytest.raises(gplk.GplkError):
        gplk.selftest_wait_timeout(10_000_000_000)
