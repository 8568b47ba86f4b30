"""FP8 E4M3 TN GEMM (tcgen05) against the double-accumulated oracle on the
same quantised operands (shapes that take every tile choice: CTA-pair
256 x 256, single-CTA 128 x 256 / 128 x 128 / 128 x 64), and against the reference's own cuBLASLt wrapper
(runner/src/gemm_lt.cu, compiled into oracle/_ref) at the 8192^3 rung.
Bar: relative Frobenius error <= 1e-2 (BF16 output)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _rel_fro(got, want):
    got = np.asarray(got, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


def _operands(oracle, M, N, K, seed):
    a = oracle.normal_f32(M * K, seed).reshape(M, K)
    b = oracle.normal_f32(N * K, seed + 1).reshape(N, K)
    qa, sa = oracle.quantize_fp8(a)
    qb, sb = oracle.quantize_fp8(b)
    return qa, sa, qb, sb


def _run(gplk, qa, sa, qb, sb, cuda):
    import torch

    M, N = qa.shape[0], qb.shape[0]
    tA = torch.from_numpy(qa).to(cuda)
    tB = torch.from_numpy(qb).to(cuda)
    D = torch.full((N, M), float("nan"), dtype=torch.bfloat16, device=cuda)
    s_a = torch.tensor([sa], dtype=torch.float32, device=cuda)
    s_b = torch.tensor([sb], dtype=torch.float32, device=cuda)
    gplk.gemm_fp8_tn(tA, tB, D, s_a, s_b)
    torch.cuda.synchronize()
    return D.float().cpu().numpy()


@pytest.mark.parametrize("mnk", [(128, 256, 128), (256, 256, 256), (512, 512, 1024), (1024, 768, 512), (300, 520, 256), (136, 264, 384),
                                 (200, 300, 512), (129, 257, 144), (1, 1, 16), (640, 1280, 2048),
                                 (4352, 264, 128),   # 1-CTA 128 x 128 tiles (too few pair tiles for one wave)
                                 (4352, 2304, 128),  # pair tiles: 17 rows, a second, one-row raster group
                                 (1536, 1536, 512), (1000, 1000, 1008),  # 1-CTA 128 x 128 / 128 x 64 tiles
                                 (2560, 2048, 256),  # 80 pair tiles: a short last wave run as 256 x 128 halves
                                 (2600, 2048, 128)])  # the same with a ragged last row of tiles
def test_fp8_full_vs_oracle(mnk, gplk, oracle, cuda):
    M, N, K = mnk
    qa, sa, qb, sb = _operands(oracle, M, N, K, seed=M * 7 + N)
    got = _run(gplk, qa, sa, qb, sb, cuda)
    want = oracle.gemm_fp8_tn(qa, qb, sa, sb)  # (N, M)
    assert np.isfinite(got).all()
    assert _rel_fro(got, want) <= TOL, mnk
    # tighter: each element within a couple of BF16 ulps of the exact value
    bf = oracle.bf16_round(want.astype(np.float32))
    assert np.max(np.abs(got - bf)) <= 2 ** -7 * np.max(np.abs(want)) + 1e-6


def test_fp8_8192_sampled_vs_oracle(gplk, oracle, cuda):
    M = N = K = 8192
    qa, sa, qb, sb = _operands(oracle, M, N, K, seed=8192)
    got = _run(gplk, qa, sa, qb, sb, cuda)
    rng = np.random.default_rng(0)
    pairs = np.stack([rng.integers(0, M, 4096), rng.integers(0, N, 4096)], axis=1)
    want = oracle.gemm_fp8_tn(qa, qb, sa, sb, pairs)
    g = got[pairs[:, 1], pairs[:, 0]]
    assert _rel_fro(g, want) <= TOL


@pytest.mark.skipif(not __import__("oracle").ref_available(), reason="reference not compiled")
@pytest.mark.parametrize("n", [1024, 8192])
def test_fp8_vs_reference_cublaslt(n, gplk, oracle, cuda):
    """The reference's own FP8 path (gpl_lt_init(FP8, n) + gpl_lt_enqueue),
    fed the identical quantised operands through its public dA/dB/scale
    pointers; D compared at <= 1e-2 relative Frobenius."""
    import torch

    L = oracle.ref_lib()
    qa, sa, qb, sb = _operands(oracle, n, n, n, seed=n + 3)
    ours = _run(gplk, qa, sa, qb, sb, cuda)
    g = L.ref_lt_new()
    stream = torch.cuda.current_stream().cuda_stream
    assert L.gpl_lt_init(g, oracle.PREC["fp8"], n, stream) == 0
    try:
        ptrs = (ctypes.c_void_p * 7)()
        L.ref_lt_ptrs(g, ptrs)
        dA, dB, _, dD, dSA, dSB, _ = [p for p in ptrs]
        torch.cuda.synchronize()
        cud = torch.cuda
        # Row m of A (K bytes) is column m of the K x M column-major matrix
        # cuBLASLt transposes (TRANSA=T): the same bytes as ours.
        tA = torch.from_numpy(qa).to(cuda)
        tB = torch.from_numpy(qb).to(cuda)
        sc = torch.tensor([sa, sb], dtype=torch.float32, device=cuda)
        import ctypes as C
        cudart = C.CDLL("libcudart.so.12")
        cudart.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
        for dst, src, nb in ((dA, tA.data_ptr(), n * n), (dB, tB.data_ptr(), n * n),
                             (dSA, sc.data_ptr(), 4), (dSB, sc.data_ptr() + 4, 4)):
            assert cudart.cudaMemcpy(dst, src, nb, 3) == 0  # device to device
        assert L.gpl_lt_enqueue(g, 1) == 0
        cud.synchronize()
        ref = torch.empty((n, n), dtype=torch.bfloat16, device=cuda)
        assert cudart.cudaMemcpy(ref.data_ptr(), dD, n * n * 2, 3) == 0
        cud.synchronize()
        ref = ref.float().cpu().numpy()  # (N, M) storage of column-major D
    finally:
        L.gpl_lt_free(g)
        L.ref_lt_delete(g)
    assert _rel_fro(ours, ref.astype(np.float64)) <= TOL


def test_fp8_rejects_bad_k(gplk, cuda):
    import torch

    A = torch.zeros(128, 24, dtype=torch.uint8, device=cuda)
    D = torch.empty(128, 128, dtype=torch.bfloat16, device=cuda)
    s = torch.ones(1, device=cuda)
    with pytest.raises(gplk.GplkError):
        gplk.gemm_fp8_tn(A, A, D, s, s)


def test_fp8_split_last_wave_is_bit_identical(gplk, oracle, cuda):
    """4096^3 on CTA pairs runs its short last wave as 256 x 128 half tiles;
    the two 4096 x 2048 column halves, computed by separate calls whose last
    wave is too full to split, must give the same bits."""
    import torch

    n = 4096
    qa, sa, qb, sb = _operands(oracle, n, n, n, seed=4243)
    A, B = torch.from_numpy(qa).to(cuda), torch.from_numpy(qb).to(cuda)
    ta = torch.tensor([sa], dtype=torch.float32, device=cuda)
    tb = torch.tensor([sb], dtype=torch.float32, device=cuda)
    full = torch.empty((n, n), dtype=torch.bfloat16, device=cuda)
    gplk.gemm_fp8_tn(A, B, full, ta, tb)
    h = n // 2
    parts = []
    for i in range(2):
        Dp = torch.empty((h, n), dtype=torch.bfloat16, device=cuda)
        gplk.gemm_fp8_tn(A, B[i * h:(i + 1) * h].contiguous(), Dp, ta, tb)
        parts.append(Dp)
    torch.cuda.synchronize()
    assert torch.equal(full.view(torch.int16), torch.cat(parts).view(torch.int16))
