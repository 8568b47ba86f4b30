"""Dense tensor-core GEMMs (gplk_gemm_{bf16,f16,tf32,i8}_nn) against the
oracle and against the reference's own cublasGemmEx rung.

Layout is the reference's (runner/src/workload_gemm.c:155-163): every
matrix column-major, C = A * B. As numpy/torch arrays: A is (K, M), B is
(N, K), D is (N, M).

Tolerances (relative Frobenius norm against the double-accumulated oracle):
  bf16  4e-3   (BF16 output rounding, 2^-9 per element)
  f16   2e-3   (FP16 output rounding, 2^-12 per element, FP32 accumulation)
  tf32  5e-3   (TF32 products carry 10 mantissa bits)
  i8    exact  (integer arithmetic)
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = {"bf16": 4e-3, "f16": 2e-3, "tf32": 5e-3}
GPL_PREC = {"fp32": 1, "tf32": 2, "f16": 3, "bf16": 4, "i8": 7}  # gpl_prec_t (runner/src/args.h:30-39)


def _inputs(prec: str, M: int, N: int, K: int, seed: int):
    """(A values, B values, A device tensor, B device tensor, D device tensor)."""
    import torch

    rng = np.random.default_rng(seed)
    if prec == "i8":
        a = rng.integers(-128, 128, size=(K, M), dtype=np.int8)
        b = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
        ta, tb = torch.from_numpy(a), torch.from_numpy(b)
        td = torch.empty((N, M), dtype=torch.int32)
    else:
        a = rng.uniform(-1.0, 1.0, size=(K, M)).astype(np.float32)
        b = rng.uniform(-1.0, 1.0, size=(N, K)).astype(np.float32)
        if prec == "bf16":
            ta = torch.from_numpy(a).to(torch.bfloat16)
            tb = torch.from_numpy(b).to(torch.bfloat16)
            a, b = ta.float().numpy(), tb.float().numpy()
            td = torch.empty((N, M), dtype=torch.bfloat16)
        elif prec == "f16":
            ta = torch.from_numpy(a).to(torch.float16)
            tb = torch.from_numpy(b).to(torch.float16)
            a, b = ta.float().numpy(), tb.float().numpy()
            td = torch.empty((N, M), dtype=torch.float16)
        else:
            ta, tb = torch.from_numpy(a), torch.from_numpy(b)
            td = torch.empty((N, M), dtype=torch.float32)
    return a, b, ta.cuda(), tb.cuda(), td.cuda()


def _rel(x: np.ndarray, ref: np.ndarray) -> float:
    return float(np.linalg.norm(x.astype(np.float64) - ref) / max(np.linalg.norm(ref), 1e-30))


# (4608, 384, 128) and (4352, 272, 64) give more than one raster group of
# 256-row pair tiles (8 per group for 2- and 4-byte operands, 16 for INT8),
# so odd groups walk N backwards, the last group ragged. (2560, 2048, 128)
# has 80 pair tiles: more than one wave of pairs, the short last wave run as
# 256 x 128 half tiles.
SHAPES = [(256, 256, 256), (1024, 1024, 1024), (512, 384, 1024), (264, 520, 128), (128, 256, 512),
          (768, 1, 64), (2048, 512, 4096), (4608, 384, 128), (4352, 272, 64), (2560, 2048, 128)]


@pytest.mark.parametrize("prec", ["bf16", "f16", "tf32", "i8"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_matches_oracle(prec, shape, gplk, oracle, cuda):
    import torch

    M, N, K = shape
    if prec == "i8" and (M % 16 or K % 16):
        pytest.skip("i8 needs M, K multiples of 16")
    a, b, ta, tb, td = _inputs(prec, M, N, K, seed=M * 7 + N * 3 + K)
    gplk.gemm_nn(prec, ta, tb, td, M, N, K)
    torch.cuda.synchronize()
    if prec == "i8":
        ref = oracle.gemm_nn_i8(a, b, M, N, K)
        assert np.array_equal(td.cpu().numpy(), ref)
    else:
        ref = oracle.gemm_nn_f64(a, b, M, N, K)
        got = td.float().cpu().numpy()
        assert _rel(got, ref) <= TOL[prec], (prec, shape, _rel(got, ref))


@pytest.mark.parametrize("prec", ["bf16", "f16", "tf32", "i8"])
def test_short_k_and_zero_fill(prec, gplk, oracle, cuda):
    """K smaller than one stage (zero-filled by TMA beyond K) and ragged N."""
    import torch

    M, N, K = 256, 300, 16 if prec != "i8" else 32
    a, b, ta, tb, td = _inputs(prec, M, N, K, seed=5)
    gplk.gemm_nn(prec, ta, tb, td, M, N, K)
    torch.cuda.synchronize()
    if prec == "i8":
        assert np.array_equal(td.cpu().numpy(), oracle.gemm_nn_i8(a, b, M, N, K))
    else:
        assert _rel(td.float().cpu().numpy(), oracle.gemm_nn_f64(a, b, M, N, K)) <= TOL[prec]


@pytest.mark.parametrize("prec", ["bf16", "f16", "tf32", "i8"])
def test_bad_arguments(prec, gplk, cuda):
    import torch

    align = {"bf16": 8, "f16": 8, "tf32": 4, "i8": 16}[prec]
    _, _, ta, tb, td = _inputs(prec, 256, 256, 256, seed=1)
    with pytest.raises(gplk.GplkError):
        gplk.gemm_nn(prec, ta[:, : 256 - align // 2].contiguous(), tb, td[:, : 256 - align // 2].contiguous(),
                     256 - align // 2, 256, 256)
    gplk.gemm_nn(prec, ta, tb, td, 256, 256, 256)  # the library still works
    torch.cuda.synchronize()


@pytest.mark.parametrize("prec", ["bf16", "f16", "tf32", "i8"])
@pytest.mark.parametrize("n", [1024, 2048])
def test_against_reference_cublas_rung(prec, n, gplk, oracle, cuda):
    """The reference's own GEMM rung call (cublasGemmEx as
    runner/src/workload_gemm.c:155-163 issues it, compiled from that file) on
    the same operands. libgplk must be at least as accurate against the
    oracle, and agree with the reference within the tolerance (bit-exact for
    i8)."""
    import torch

    if not oracle.ref_available():
        pytest.skip("reference library not built")
    a, b, ta, tb, td = _inputs(prec, n, n, n, seed=n + 11)
    tr = torch.empty_like(td)
    gplk.gemm_nn(prec, ta, tb, td, n, n, n)
    st = oracle.ref_lib().ref_gemm_ex(GPL_PREC[prec], ta.data_ptr(), tb.data_ptr(), tr.data_ptr(), n,
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    if st != 0:
        pytest.skip(f"the reference's cublasGemmEx rejects {prec} here (status {st})")
    if prec == "i8":
        assert np.array_equal(td.cpu().numpy(), tr.cpu().numpy())
        return
    ref = oracle.gemm_nn_f64(a, b, n, n, n)
    ours, theirs = td.float().cpu().numpy(), tr.float().cpu().numpy()
    e_ours, e_ref = _rel(ours, ref), _rel(theirs, ref)
    print(f"{prec} n={n}: rel err gplk {e_ours:.2e}, reference {e_ref:.2e}")
    assert e_ours <= max(TOL[prec], 1.05 * e_ref)
    assert _rel(ours, theirs.astype(np.float64)) <= max(2 * TOL[prec], 2 * e_ref)


def _old_d(prec: str, M: int, N: int, seed: int):
    """(values as float64 / int64, device tensor) of a random old D."""
    import torch

    rng = np.random.default_rng(seed)
    if prec == "i8":
        v = rng.integers(-(1 << 31), 1 << 31, size=(N, M), dtype=np.int64).astype(np.int32)
        return v.astype(np.int64), torch.from_numpy(v).cuda()
    v = rng.uniform(-16.0, 16.0, size=(N, M)).astype(np.float32)
    t = torch.from_numpy(v).to({"bf16": torch.bfloat16, "f16": torch.float16, "tf32": torch.float32}[prec])
    return t.float().numpy().astype(np.float64), t.cuda()


@pytest.mark.parametrize("prec", ["bf16", "f16", "tf32", "i8"])
@pytest.mark.parametrize("shape", [(256, 256, 256), (1024, 1024, 1024), (264, 520, 128), (768, 1, 64),
                                   (4352, 272, 64), (2560, 2048, 64)], ids=lambda s: "x".join(map(str, s)))
def test_accumulate_matches_oracle(prec, shape, gplk, oracle, cuda):
    """beta = 1 (the tensor stream's C = A * B + C): the old D is read and the
    product added before the single rounding; S32 wraps."""
    import torch

    M, N, K = shape
    if prec == "i8" and (M % 16 or K % 16):
        pytest.skip("i8 needs M, K multiples of 16")
    a, b, ta, tb, _ = _inputs(prec, M, N, K, seed=M + 5 * N + K)
    d0, td = _old_d(prec, M, N, seed=M * 3 + K)
    gplk.gemm_nn(prec, ta, tb, td, M, N, K, accumulate=True)
    torch.cuda.synchronize()
    if prec == "i8":
        want = ((oracle.gemm_nn_i8(a, b, M, N, K).astype(np.int64) + d0 + (1 << 31)) % (1 << 32) - (1 << 31))
        assert np.array_equal(td.cpu().numpy().astype(np.int64), want)
    else:
        want = oracle.gemm_nn_f64(a, b, M, N, K) + d0
        assert _rel(td.float().cpu().numpy(), want) <= TOL[prec], (prec, shape)


@pytest.mark.parametrize("prec", ["bf16", "f16", "tf32", "i8"])
def test_accumulate_vs_reference_tensor_stream(prec, gplk, oracle, cuda):
    """The reference rung's own tensor stream (tensor_stream_init /
    tensor_stream_enqueue, runner/src/workload_powervirus.cu:281-397, compiled
    from that file): two beta = 1 GEMMs into the same C on the same operands.
    INT8 bit-exact; otherwise libgplk at least as close to the
    double-accumulated oracle as the reference (whose FP16 path accumulates in
    FP16 under CUBLAS_TENSOR_OP_MATH)."""
    import torch

    from gplk.lt import device_view

    if not oracle.ref_available():
        pytest.skip("reference library not built")
    n = 1024
    a, b, ta, tb, _ = _inputs(prec, n, n, n, seed=77)
    d0, td = _old_d(prec, n, n, seed=78)
    ref_c = td.clone()
    for _ in range(2):
        gplk.gemm_nn(prec, ta, tb, td, n, n, n, accumulate=True)
    L = oracle.ref_lib()
    r = L.ref_ts_new(GPL_PREC[prec], n)
    assert r, "reference tensor stream set-up failed"
    try:
        ptrs = (ctypes.c_void_p * 4)()
        L.ref_ts_ptrs(r, ptrs)
        nb_in, nb_out = ta.numel() * ta.element_size(), ref_c.numel() * ref_c.element_size()
        device_view(ptrs[0], nb_in).copy_(ta.view(-1).view(torch.uint8))
        device_view(ptrs[1], nb_in).copy_(tb.view(-1).view(torch.uint8))
        device_view(ptrs[2], nb_out).copy_(ref_c.view(-1).view(torch.uint8))
        torch.cuda.synchronize()
        L.ref_ts_enqueue(r, 2)
        torch.cuda.synchronize()
        theirs_t = device_view(ptrs[2], nb_out).clone().view(ref_c.dtype).view(n, n)
    finally:
        L.ref_ts_delete(r)
    torch.cuda.synchronize()
    if prec == "i8":
        assert torch.equal(td, theirs_t)
        return
    want = 2.0 * oracle.gemm_nn_f64(a, b, n, n, n) + d0
    e_ours = _rel(td.float().cpu().numpy(), want)
    e_ref = _rel(theirs_t.float().cpu().numpy(), want)
    print(f"{prec} beta=1 x2: rel err gplk {e_ours:.2e}, reference tensor stream {e_ref:.2e}")
    assert e_ours <= max(TOL[prec], 1.05 * e_ref)
