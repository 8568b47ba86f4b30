"""The device-side operand quantisers (gplk.operands) against the oracle's C
restatement of the same rules, byte for byte, on CPU tensors (and on the
GPU under -m gpu)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gplk import operands as O


def _inputs(oracle, rows, k, seed):
    x = oracle.normal_f32(rows * k, seed).reshape(rows, k)
    # Scale some rows to reach E4M3 subnormal block scales and E2M1 ties.
    x[1] *= 1e-3
    x[2, :16] = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, -0.25, -0.75, -1.25, -1.75, -2.5, -3.5, -5.0, 0.0]
    x[3, :16] = 0.0
    return x


@pytest.mark.parametrize("rows,k", [(1, 16), (7, 48), (130, 80), (256, 512)])
def test_nvfp4_matches_oracle(oracle, rows, k):
    x = oracle.normal_f32(rows * k, 11).reshape(rows, k) if rows < 4 else _inputs(oracle, rows, k, 11)
    want_q, want_sf, want_g = oracle.quantize_nvfp4(x)
    q, sf, g = O.quantize_nvfp4(torch.from_numpy(x))
    assert np.float32(g) == np.float32(want_g)
    assert sf.numel() == O.sf_bytes(rows, k) == oracle.sf_bytes(rows, k)
    assert np.array_equal(sf.numpy(), want_sf)
    assert np.array_equal(q.numpy(), want_q)


def test_e2m1_ties_and_saturation(oracle):
    v = np.array([0.0, -0.0, 0.2, 0.25, 0.26, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.1, 6.0, 7.0, 1e9, -1e9,
                  float("nan")], dtype=np.float32)
    got = O.e2m1_codes(torch.from_numpy(v)).numpy()
    want = [oracle.e2m1_encode(float(t)) for t in v]
    assert list(got) == want


@pytest.mark.parametrize("n", [1, 1000, 65536])
def test_fp8_matches_oracle(oracle, n):
    x = oracle.normal_f32(n, 5)
    x[: min(n, 4)] *= 1e-4  # subnormal codes
    want_q, want_s = oracle.quantize_fp8(x)
    q, s = O.quantize_fp8(torch.from_numpy(x))
    assert np.float32(s) == np.float32(want_s)
    assert np.array_equal(q.numpy(), want_q)


def test_sf_layout_positions(oracle):
    rows, kb_n = 300, 9
    s8 = torch.arange(rows * kb_n, dtype=torch.int64).remainder(251).add(1).to(torch.uint8).view(rows, kb_n)
    flat = O.sf_layout(s8).numpy()
    for r in (0, 31, 32, 127, 128, 200, 299):
        for kb in range(kb_n):
            assert flat[oracle.sf_offset(r, kb, kb_n)] == int(s8[r, kb])


@pytest.mark.gpu
def test_quantisers_on_device_match_oracle(oracle, cuda):
    x = _inputs(oracle, 384, 1024, 3)
    want_q, want_sf, want_g = oracle.quantize_nvfp4(x)
    q, sf, g = O.quantize_nvfp4(torch.from_numpy(x).to(cuda))
    assert np.float32(g) == np.float32(want_g)
    assert np.array_equal(sf.cpu().numpy(), want_sf)
    assert np.array_equal(q.cpu().numpy(), want_q)
    wq, ws = oracle.quantize_fp8(x)
    q8, s8 = O.quantize_fp8(torch.from_numpy(x).to(cuda))
    assert np.float32(s8) == np.float32(ws)
    assert np.array_equal(q8.cpu().numpy(), wq)
