"""The oracle pinned against the reference and the golden fixtures (CPU)."""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_e4m3_decode_matches_torch_table(oracle):
    g = json.loads((GOLDEN / "e4m3.json").read_text())
    ours = oracle.e4m3_decode_table()
    for code, want in enumerate(g["decode"]):
        if want is None:
            assert math.isnan(ours[code]), code
        else:
            assert ours[code] == np.float32(want), (code, ours[code], want)


def test_e4m3_encode_matches_torch(oracle):
    g = json.loads((GOLDEN / "e4m3.json").read_text())
    got = [oracle.e4m3_encode(x) for x in g["encode_in"]]
    bad = [(x, a, b) for x, a, b in zip(g["encode_in"], got, g["encode_out"]) if a != b]
    assert not bad, bad[:10]


def test_e4m3_saturates_and_round_trips(oracle):
    dec = oracle.e4m3_decode_table()
    for code in range(256):
        if code & 0x7F == 0x7F:
            continue
        assert oracle.e4m3_encode(dec[code]) == (code if dec[code] != 0 or code == 0 else code)
    assert oracle.e4m3_encode(1e9) == 0x7E
    assert oracle.e4m3_encode(-1e9) == 0xFE


def test_e2m1_grid_ties_and_saturation(oracle):
    dec = oracle.e2m1_decode_table()
    assert list(dec[:8]) == [0, 0.5, 1, 1.5, 2, 3, 4, 6]
    for code in range(16):
        if code == 8:  # -0 encodes back to -0
            assert oracle.e2m1_encode(-0.0) == 8
            continue
        assert oracle.e2m1_encode(dec[code]) == code
    # ties to even mantissa
    assert oracle.e2m1_encode(0.25) == 0
    assert oracle.e2m1_encode(0.75) == 2
    assert oracle.e2m1_encode(1.25) == 2
    assert oracle.e2m1_encode(1.75) == 4
    assert oracle.e2m1_encode(2.5) == 4
    assert oracle.e2m1_encode(3.5) == 6
    assert oracle.e2m1_encode(5.0) == 6
    assert oracle.e2m1_encode(100.0) == 7
    assert oracle.e2m1_encode(-100.0) == 15


def test_role_map_matches_reference_fixture(oracle):
    for case in json.loads((GOLDEN / "role_maps.json").read_text()):
        w = list(case["weights"])
        if case["tensor_cublas"]:
            w[0] = 0  # the reference drops the in-kernel tensor role with the cuBLAS backend
        m, c = oracle.role_map(w)
        assert m.tolist() == case["map"], case
        assert c.tolist() == case["counts"], case


@pytest.mark.skipif(not (Path(__file__).resolve().parent.parent / "oracle/_ref/libgpl_ref.so").exists(),
                    reason="reference not compiled here")
def test_role_map_matches_reference_live(oracle):
    rng = np.random.default_rng(7)
    for _ in range(300):
        w = rng.integers(0, 12, 8) * (rng.random(8) < 0.6)
        m, c = oracle.role_map(w)
        rm, rc = oracle.ref_role_map(w)
        assert m.tolist() == rm.tolist() and c.tolist() == rc.tolist(), w


def test_accounting_matches_reference(oracle):
    for case in json.loads((GOLDEN / "accounting.json").read_text()):
        op = oracle.OP[case["op"]]
        assert oracle.flops_per_iter(op, case["size"]) == case["flops"]
        assert oracle.bytes_per_iter(op, case["size"]) == case["bytes"]


def test_generators_are_seeded_and_shaped(oracle):
    a = oracle.uniform_f32(100_003, seed=0, lo=-1.0, hi=1.0)
    b = oracle.uniform_f32(100_003, seed=0, lo=-1.0, hi=1.0)
    assert np.array_equal(a, b)
    assert a.min() >= -1.0 and a.max() < 1.0
    assert abs(float(a.mean())) < 0.01
    z = oracle.normal_f32(200_001, seed=3)
    assert abs(float(z.mean())) < 0.01 and abs(float(z.std()) - 1.0) < 0.01
    assert not np.array_equal(oracle.uniform_f32(64, 1), oracle.uniform_f32(64, 2))


def test_triad_is_fmaf(oracle):
    b = oracle.uniform_f32(4099, 1)
    c = oracle.uniform_f32(4099, 2)
    a = oracle.triad_f32(b, c, 3.0)
    # fmaf(s, c, b) equals the float64 product-sum rounded once to float32
    # when the product is exact in double (24 + 24 bits <= 53).
    ref = (np.float64(3.0) * c.astype(np.float64) + b.astype(np.float64)).astype(np.float32)
    assert np.array_equal(a, ref)


def test_sgemm_oracle_small(oracle):
    rng = np.random.default_rng(0)
    A = rng.uniform(-1, 1, (37, 53)).astype(np.float32)
    B = rng.uniform(-1, 1, (53, 29)).astype(np.float32)
    C = oracle.sgemm_f64acc(A, B)
    assert np.allclose(C, A.astype(np.float64) @ B.astype(np.float64), rtol=0, atol=1e-12)


def test_fp8_quantise_and_gemm_oracle(oracle):
    x = oracle.normal_f32(64 * 96, 11).reshape(64, 96)
    q, s = oracle.quantize_fp8(x)
    assert s == pytest.approx(np.abs(x).max() / 448.0)
    lut = oracle.e4m3_decode_table()
    deq = lut[q] * s
    assert np.max(np.abs(deq - x)) <= np.abs(x).max() * 2.0 ** -3  # 3 mantissa bits
    y = oracle.normal_f32(48 * 96, 12).reshape(48, 96)
    qy, sy = oracle.quantize_fp8(y)
    D = oracle.gemm_fp8_tn(q, qy, s, sy)  # (N, M) = column-major M x N
    ref = (lut[q].astype(np.float64) @ lut[qy].astype(np.float64).T) * s * sy
    assert np.allclose(D.T, ref, rtol=1e-12, atol=1e-9)
    pairs = np.array([[0, 0], [63, 47], [5, 17]])
    assert np.allclose(oracle.gemm_fp8_tn(q, qy, s, sy, pairs), [D[n, m] for m, n in pairs])


def test_nvfp4_quantise_layout_and_gemm_oracle(oracle):
    rows, k = 200, 320
    x = oracle.normal_f32(rows * k, 5).reshape(rows, k)
    packed, sf, g = oracle.quantize_nvfp4(x)
    assert sf.size == ((rows + 127) // 128) * ((k // 16 + 3) // 4) * 512
    assert g == pytest.approx(np.abs(x).max() / (6 * 448))
    # dequantise through the documented layout and compare with x
    e2 = oracle.e2m1_decode_table()
    e4 = oracle.e4m3_decode_table()
    lo, hi = packed & 15, packed >> 4
    vals = np.empty((rows, k), np.float32)
    vals[:, 0::2], vals[:, 1::2] = e2[lo], e2[hi]
    kb_n = k // 16
    for r in (0, 31, 32, 127, 128, 199):
        for kb in range(kb_n):
            off = ((r // 128) * ((kb_n + 3) // 4) + kb // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4
            assert off == oracle.sf_offset(r, kb, kb_n)
            scale = e4[sf[off]] * g
            blk = x[r, kb * 16:(kb + 1) * 16]
            deq = vals[r, kb * 16:(kb + 1) * 16] * scale
            # the widest E2M1 step (4 -> 6) is 2 * scale, so rounding costs at
            # most one scale; a scale rounded below bmax/6 adds saturation
            bmax = float(np.abs(blk).max())
            bound = scale + max(0.0, bmax - 6 * scale) + 1e-6
            assert np.max(np.abs(deq - blk)) <= bound
    y = oracle.normal_f32(136 * k, 6).reshape(136, k)
    pb, sfb, gb = oracle.quantize_nvfp4(y)
    D = oracle.gemm_nvfp4_tn(packed, pb, sf, sfb, k, g * gb)
    # same product via explicit dequantised matrices
    def deq_all(p, s, n_rows, gg):
        v = np.empty((n_rows, k), np.float64)
        v[:, 0::2], v[:, 1::2] = e2[p & 15], e2[p >> 4]
        for r in range(n_rows):
            for kb in range(kb_n):
                v[r, kb * 16:(kb + 1) * 16] *= e4[s[oracle.sf_offset(r, kb, kb_n)]]
        return v
    ref = deq_all(packed, sf, rows, g) @ deq_all(pb, sfb, 136, gb).T * (g * gb)
    assert np.allclose(D.T, ref, rtol=1e-6, atol=1e-9)  # alpha is passed as float32


def test_powervirus_chains(oracle):
    # INT32 role: exact modular arithmetic, restated in Python integers.
    def lcg(lane, steps):
        i0, i1, i2, i3 = (0x9E3779B9 + lane) & 0xFFFFFFFF, 0x85EBCA6B, 0xC2B2AE35, 0x27D4EB2F
        for _ in range(steps):
            i0 = (i0 * 1664525 + 1013904223) & 0xFFFFFFFF
            i1 = (i1 * 22695477 + 1) & 0xFFFFFFFF
            i2 = (i2 * 1103515245 + 12345) & 0xFFFFFFFF
            i3 = (i3 * 214013 + 2531011) & 0xFFFFFFFF
        return i0 ^ i1 ^ i2 ^ i3
    for lane in (0, 7, 31):
        assert oracle.lcg_chain(lane, 1000) == lcg(lane, 1000)
    # FMA role converges to the fixed point c / (1 - m) = 1e-3.
    v = oracle.fma_chain(0, 200_000)
    assert abs(v / 8 - 1e-7 / (1 - 0.9999)) < 1e-4


def test_bf16_round(oracle):
    x = np.array([1.0, 1.00390625, 1.01171875, -3.140625, 65504.0, 1e-40], np.float32)
    import torch
    want = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(oracle.bf16_round(x), want)
