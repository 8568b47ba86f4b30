"""FP32 SGEMM on the GPU against the double-accumulated host triple loop
(tolerance 1e-5 relative, Frobenius and max-norm)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _rel_fro(got, want):
    return float(np.linalg.norm(got.astype(np.float64) - want) / max(np.linalg.norm(want), 1e-300))


def _run(gplk, A, B, cuda):
    import torch

    tA, tB = torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda)
    C = torch.full((A.shape[0], B.shape[1]), float("nan"), device=cuda)
    gplk.sgemm(tA, tB, C)
    torch.cuda.synchronize()
    return C.cpu().numpy()


def test_sgemm_1024_seed0(gplk, oracle, cuda):
    n = 1024
    A = oracle.uniform_f32(n * n, seed=0, lo=-1.0, hi=1.0).reshape(n, n)
    B = oracle.uniform_f32(n * n, seed=1, lo=-1.0, hi=1.0).reshape(n, n)
    got = _run(gplk, A, B, cuda)
    want = oracle.sgemm_f64acc(A, B)
    assert _rel_fro(got, want) <= TOL
    assert float(np.max(np.abs(got - want))) <= TOL * float(np.max(np.abs(want)))


# (2048, 2304, 300) and (2000, 2300, 200) fill two whole waves of 128 x 128
# tiles (one tile per block, 8 x 16 per thread, ragged edges in the second);
# (1000, 1000, 333), (768, 1024, 1024) and (1024, 2048, 4096) run stream-K.
@pytest.mark.parametrize("mnk", [(1, 1, 1), (33, 17, 5), (100, 130, 257), (257, 129, 1000),
                                 (64, 64, 16), (128, 256, 64), (2048, 512, 300), (3000, 2000, 128),
                                 (1000, 1000, 333), (768, 1024, 1024), (1024, 2048, 4096),
                                 (2048, 2304, 300), (2000, 2300, 200)])
def test_sgemm_shapes(mnk, gplk, oracle, cuda):
    M, N, K = mnk
    A = oracle.uniform_f32(M * K, seed=M, lo=-1.0, hi=1.0).reshape(M, K)
    B = oracle.uniform_f32(K * N, seed=N + 7, lo=-1.0, hi=1.0).reshape(K, N)
    got = _run(gplk, A, B, cuda)
    want = oracle.sgemm_f64acc(A, B)
    assert _rel_fro(got, want) <= TOL, mnk


def test_sgemm_strided_views(gplk, oracle, cuda):
    import torch

    M, N, K = 200, 120, 96
    big = torch.from_numpy(oracle.uniform_f32(M * (K + 8), 3, -1, 1).reshape(M, K + 8)).to(cuda)
    A = big[:, :K]  # lda = K + 8
    B = torch.from_numpy(oracle.uniform_f32(K * N, 4, -1, 1).reshape(K, N)).to(cuda)
    C = torch.empty(M, N, device=cuda)
    gplk.sgemm(A, B, C)
    torch.cuda.synchronize()
    want = oracle.sgemm_f64acc(np.ascontiguousarray(A.cpu().numpy()), B.cpu().numpy())
    assert _rel_fro(C.cpu().numpy(), want) <= TOL


def test_sgemm_k_zero_writes_zeros(gplk, cuda):
    import torch

    A = torch.empty(8, 0, device=cuda)
    B = torch.empty(0, 8, device=cuda)
    C = torch.full((8, 8), 5.0, device=cuda)
    gplk.sgemm(A, B, C)
    torch.cuda.synchronize()
    assert torch.count_nonzero(C) == 0


def test_sgemm_matches_cublas_fp32(gplk, oracle, cuda):
    """Cross-check against cuBLAS in true FP32 (TF32 off), the library the
    reference's sgemm rung calls."""
    import torch

    torch.backends.cuda.matmul.allow_tf32 = False
    n = 1024
    A = torch.from_numpy(oracle.uniform_f32(n * n, 0, -1, 1).reshape(n, n)).to(cuda)
    B = torch.from_numpy(oracle.uniform_f32(n * n, 1, -1, 1).reshape(n, n)).to(cuda)
    C = torch.empty(n, n, device=cuda)
    gplk.sgemm(A, B, C)
    ref = A @ B
    torch.cuda.synchronize()
    rel = (torch.linalg.norm((C - ref).double()) / torch.linalg.norm(ref.double())).item()
    assert rel <= TOL


def test_sgemm_matches_reference_rung_call(gplk, oracle, cuda):
    """The reference rung's own call: cublasGemmEx COMPUTE_32F, DEFAULT_MATH,
    column-major NN (runner/src/workload_gemm.c:155-163, built from that file
    into the reference library). Column-major C = A * B is the row-major
    product C^T = B^T A^T, so the row-major gplk SGEMM of (B, A) gives the
    same bytes."""
    import ctypes

    import torch

    if not oracle.ref_available():
        pytest.skip("reference library not built")
    n = 1024
    A = torch.from_numpy(oracle.uniform_f32(n * n, 0, -1, 1).reshape(n, n)).to(cuda)
    B = torch.from_numpy(oracle.uniform_f32(n * n, 1, -1, 1).reshape(n, n)).to(cuda)
    C = torch.empty(n, n, device=cuda)
    R = torch.empty(n, n, device=cuda)
    gplk.sgemm(B, A, C)  # row-major (B A) = column-major (A B) with these buffers
    st = oracle.ref_lib().ref_gemm_ex(1, A.data_ptr(), B.data_ptr(), R.data_ptr(), n,
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert st == 0
    rel = (torch.linalg.norm((C - R).double()) / torch.linalg.norm(R.double())).item()
    assert rel <= TOL, rel


def test_sgemm_stream_k_repeatable_and_per_stream(gplk, oracle, cuda):
    """Shapes whose 128 x 128 tiles leave the last wave ragged run stream-K
    (partial tiles parked in a per-stream workspace, flags carrying a launch
    epoch). Back-to-back calls with new inputs, and calls on two streams at
    once, must each be exact to the tolerance and bit-identical run to run."""
    import torch

    M, N, K = 2048, 2048, 2048  # 256 tiles on 148 SMs: stream-K
    gplk.status_read()  # start from a clear device status word
    ins = [(oracle.uniform_f32(M * K, seed=20 + i, lo=-1.0, hi=1.0).reshape(M, K),
            oracle.uniform_f32(K * N, seed=40 + i, lo=-1.0, hi=1.0).reshape(K, N)) for i in range(2)]
    want = [oracle.sgemm_f64acc(A, B) for A, B in ins]
    dev = [(torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda)) for A, B in ins]
    outs = [torch.full((M, N), float("nan"), device=cuda) for _ in range(4)]
    for r in range(2):  # same stream: first operand pair, second, first again
        gplk.sgemm(dev[0][0], dev[0][1], outs[0])
        gplk.sgemm(dev[1][0], dev[1][1], outs[1])
        gplk.sgemm(dev[0][0], dev[0][1], outs[2])
    torch.cuda.synchronize()
    s1, s2 = torch.cuda.Stream(device=cuda), torch.cuda.Stream(device=cuda)
    with torch.cuda.stream(s1):
        gplk.sgemm(dev[0][0], dev[0][1], outs[3], stream=s1)
    with torch.cuda.stream(s2):
        gplk.sgemm(dev[1][0], dev[1][1], outs[1], stream=s2)
    torch.cuda.synchronize()
    got = [o.cpu().numpy() for o in outs]
    assert _rel_fro(got[0], want[0]) <= TOL
    assert _rel_fro(got[1], want[1]) <= TOL
    assert np.array_equal(got[0], got[2]) and np.array_equal(got[0], got[3])
    assert gplk.status_read() == (0, 0)


# beta = 1 (C = A B + C, the fp32 powervirus tensor stream's call) on every
# kernel family: stream-K (1024^3, 1000 x 1000 x 333), whole tiles (2048 x
# 2304 x 300), the register-staged kernels (100 x 130 x 257, unaligned), and
# the split-K cluster pair (257 x 129 x 1000).
@pytest.mark.parametrize("mnk", [(1024, 1024, 1024), (1000, 1000, 333), (2048, 2304, 300), (100, 130, 257),
                                 (257, 129, 1000), (33, 17, 5)])
@pytest.mark.parametrize("beta", [1.0, 0.5])
def test_sgemm_beta(mnk, beta, gplk, oracle, cuda):
    import torch

    M, N, K = mnk
    A = oracle.uniform_f32(M * K, seed=M + 1, lo=-1.0, hi=1.0).reshape(M, K)
    B = oracle.uniform_f32(K * N, seed=N + 2, lo=-1.0, hi=1.0).reshape(K, N)
    C0 = oracle.uniform_f32(M * N, seed=K + 3, lo=-8.0, hi=8.0).reshape(M, N)
    C = torch.from_numpy(C0).to(cuda)
    gplk.sgemm(torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda), C, beta=beta)
    torch.cuda.synchronize()
    want = oracle.sgemm_f64acc(A, B) + beta * C0.astype(np.float64)
    assert _rel_fro(C.cpu().numpy(), want) <= TOL, mnk


def test_sgemm_workspace_optional(gplk, oracle, cuda):
    """A stream-K shape with the caller's workspace, with none, and with one
    too small (the whole-tile kernel then runs): all within the tolerance;
    no workspace and a too-small one take the same kernel, bit for bit."""
    import torch

    n = 1024
    assert gplk.sgemm_workspace_bytes(n, n, n) > 0        # 64 tiles on 148 SMs: stream-K
    assert gplk.sgemm_workspace_bytes(4096, 4096, 4096) == 0  # whole waves: no workspace
    A = oracle.uniform_f32(n * n, seed=0, lo=-1.0, hi=1.0).reshape(n, n)
    B = oracle.uniform_f32(n * n, seed=1, lo=-1.0, hi=1.0).reshape(n, n)
    tA, tB = torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda)
    want = oracle.sgemm_f64acc(A, B)
    ws = torch.empty(gplk.sgemm_workspace_bytes(n, n, n), dtype=torch.uint8, device=cuda)
    small = torch.empty(4096, dtype=torch.uint8, device=cuda)
    outs = [torch.full((n, n), float("nan"), device=cuda) for _ in range(3)]
    gplk.sgemm(tA, tB, outs[0], workspace=ws)
    gplk.sgemm(tA, tB, outs[1], workspace=None)
    gplk.sgemm(tA, tB, outs[2], workspace=small)
    torch.cuda.synchronize()
    got = [o.cpu().numpy() for o in outs]
    for g in got:
        assert _rel_fro(g, want) <= TOL
    assert np.array_equal(got[1], got[2])
    assert gplk.status_read() == (0, 0)
