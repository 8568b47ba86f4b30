"""NVFP4 block-scaled GEMM (tcgen05 kind::mxf4nvf4, UE4M3 scale per 16
K-elements) against the double-accumulated oracle on the same quantised
operands and scale bytes. Bar: relative Frobenius error <= 1e-2."""
from __future__ import annotations

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
    pa, sfa, ga = oracle.quantize_nvfp4(a)
    pb, sfb, gb = oracle.quantize_nvfp4(b)
    return pa, sfa, pb, sfb, ga * gb


def _run(gplk, pa, sfa, pb, sfb, alpha, K, cuda):
    import torch

    M, N = pa.shape[0], pb.shape[0]
    t = lambda x: torch.from_numpy(x).to(cuda)
    D = torch.full((N, M), float("nan"), dtype=torch.bfloat16, device=cuda)
    al = torch.tensor([alpha], dtype=torch.float32, device=cuda)
    gplk.gemm_nvfp4_tn(t(pa), t(pb), t(sfa), t(sfb), D, K, al)
    torch.cuda.synchronize()
    return D.float().cpu().numpy()


@pytest.mark.parametrize("mnk", [(128, 256, 256), (256, 256, 512), (512, 768, 1024), (128, 384, 512),
                                 (200, 300, 256), (1024, 1024, 2048), (384, 512, 768), (136, 264, 1280)])
def test_nvfp4_full_vs_oracle(mnk, gplk, oracle, cuda):
    M, N, K = mnk
    pa, sfa, pb, sfb, alpha = _operands(oracle, M, N, K, seed=M + 3 * N)
    got = _run(gplk, pa, sfa, pb, sfb, alpha, K, cuda)
    want = oracle.gemm_nvfp4_tn(pa, pb, sfa, sfb, K, alpha)
    assert np.isfinite(got).all()
    assert _rel_fro(got, want) <= TOL, mnk
    bf = oracle.bf16_round(want.astype(np.float32))
    assert np.max(np.abs(got - bf)) <= 2 ** -7 * np.max(np.abs(want)) + 1e-6


@pytest.mark.parametrize("n", [2048, 4096, 8192, 16384])
def test_nvfp4_ladder_sampled_vs_oracle(n, gplk, oracle, cuda):
    pa, sfa, pb, sfb, alpha = _operands(oracle, n, n, n, seed=n)
    got = _run(gplk, pa, sfa, pb, sfb, alpha, n, cuda)
    rng = np.random.default_rng(n)
    pairs = np.stack([rng.integers(0, n, 2048), rng.integers(0, n, 2048)], axis=1)
    want = oracle.gemm_nvfp4_tn(pa, pb, sfa, sfb, n, alpha, pairs)
    assert _rel_fro(got[pairs[:, 1], pairs[:, 0]], want) <= TOL


@pytest.mark.parametrize("mnk", [(4096, 2048, 256), (2048, 4352, 512), (2560, 2304, 768), (2600, 2304, 512)])
def test_nvfp4_several_tiles_per_cta_short_k(mnk, gplk, oracle, cuda):
    """More tiles than SMs, so each persistent CTA hands its accumulator from
    tile to tile, with K of only 1 to 3 pipeline stages per tile. The last
    two shapes leave a last wave of at most half the CTAs (180 and 189 tiles
    on 148 SMs), which runs as 128-column half tiles; the last has a ragged
    final row of tiles (M = 2600)."""
    M, N, K = mnk
    pa, sfa, pb, sfb, alpha = _operands(oracle, M, N, K, seed=M + N + K)
    got = _run(gplk, pa, sfa, pb, sfb, alpha, K, cuda)
    assert np.isfinite(got).all()
    rng = np.random.default_rng(K)
    pairs = np.stack([rng.integers(0, M, 4096), rng.integers(0, N, 4096)], axis=1)
    want = oracle.gemm_nvfp4_tn(pa, pb, sfa, sfb, K, alpha, pairs)
    assert _rel_fro(got[pairs[:, 1], pairs[:, 0]], want) <= TOL


def test_nvfp4_rejects_bad_k(gplk, cuda):
    import torch

    A = torch.zeros(128, 64, dtype=torch.uint8, device=cuda)  # K = 128
    sf = torch.zeros(4096, dtype=torch.uint8, device=cuda)
    D = torch.empty(128, 128, dtype=torch.bfloat16, device=cuda)
    al = torch.ones(1, device=cuda)
    with pytest.raises(gplk.GplkError):
        gplk.gemm_nvfp4_tn(A, A, sf, sf, D, 128, al)


@pytest.mark.parametrize("n", [2048, 4096, 8192, 16384])
def test_nvfp4_vs_cublaslt(n, gplk, oracle, cuda):
    """The NVFP4 ladder against cuBLASLt's NVFP4 GEMM (VEC16_UE4M3 block
    scales, the configuration runner/src/gemm_lt.cu lacks) on identical
    operands and scale bytes: relative Frobenius error <= 1e-2 over all of D."""
    import torch

    pa, sfa, pb, sfb, alpha = _operands(oracle, n, n, n, seed=n + 1)
    ours = _run(gplk, pa, sfa, pb, sfb, alpha, n, cuda)
    t = lambda x: torch.from_numpy(x).to(cuda)
    ref = torch.empty((n, n), dtype=torch.bfloat16, device=cuda)
    ws = torch.empty(32 << 20, dtype=torch.uint8, device=cuda)
    tA, tB, tSA, tSB = t(pa), t(pb), t(sfa), t(sfb)
    rc = oracle.lt_lib().oracle_lt_gemm_nvfp4_tn(
        tA.data_ptr(), tB.data_ptr(), tSA.data_ptr(), tSB.data_ptr(), ref.data_ptr(), n, n, n, alpha,
        ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    ref = ref.float().cpu().numpy().astype(np.float64)
    assert _rel_fro(ours, ref) <= TOL


def test_nvfp4_split_last_wave_is_bit_identical(gplk, oracle, cuda):
    """4096^3 runs its short last wave as 128-column half tiles; two calls
    of 4096 x 2048 (256 tiles each: a last wave too full to split) give the
    same columns without the split. The bits must agree: every output
    element sums its K-blocks in the same order."""
    import torch

    n = 4096
    pa, sfa, pb, sfb, alpha = _operands(oracle, n, n, n, seed=4242)
    t = lambda x: torch.from_numpy(x).to(cuda)
    A, SA, B, SB = t(pa), t(sfa), t(pb), t(sfb)
    al = torch.tensor([alpha], dtype=torch.float32, device=cuda)
    full = torch.empty((n, n), dtype=torch.bfloat16, device=cuda)
    gplk.gemm_nvfp4_tn(A, B, SA, SB, full, n, al)
    h = n // 2
    sf_half = SB.numel() // 2  # row blocks 0..15, then 16..31
    parts = []
    for i in range(2):
        Dp = torch.empty((h, n), dtype=torch.bfloat16, device=cuda)
        gplk.gemm_nvfp4_tn(A, B[i * h:(i + 1) * h].contiguous(), SA,
                           SB[i * sf_half:(i + 1) * sf_half].contiguous(), Dp, n, al)
        parts.append(Dp)
    torch.cuda.synchronize()
    assert torch.equal(full.view(torch.int16), torch.cat(parts).view(torch.int16))
