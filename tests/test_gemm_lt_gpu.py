"""The runner's GEMM handle (include/gemm_lt.h) as callers use it: libgplk's
gpl_lt_init, operands seeded through the struct's public dA / dB / scale
fields, gpl_lt_enqueue, the result read from dD.

FP8: compared with the reference's own gpl_lt_init / gpl_lt_enqueue
(runner/src/gemm_lt.cu:57-179, compiled into oracle/_ref) fed the same bytes
through its own struct, and with the CPU oracle on sampled entries. FP4: the
reference's path sets no block scales and cannot run, so the cuBLASLt NVFP4
harness (VEC16_UE4M3 scales) and the CPU oracle stand in for it. Bar:
relative Frobenius error <= 1e-2. The struct layout itself is checked on CPU
against the header.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
TOL = 1e-2


def _rel_fro(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


def test_struct_layout_matches_header(tmp_path):
    from gplk.lt import LtGemm

    src = tmp_path / "layout.c"
    fields = [f for f, _ in LtGemm._fields_]
    body = "".join(f'printf("%zu\\n", offsetof(gpl_lt_gemm_t, {f}));' for f in fields)
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"gemm_lt.h\"\n"
                   f"int main(void) {{ {body} printf(\"%zu\\n\", sizeof(gpl_lt_gemm_t)); return 0; }}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=gnu11", f"-I{REPO / 'include'}", "-I/usr/local/cuda/include", str(src), "-o",
                    str(exe)], check=True, capture_output=True, text=True)
    got = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    want = [getattr(LtGemm, f).offset for f in fields] + [ctypes.sizeof(LtGemm)]
    assert got == want


def _seed(view, src):
    view.copy_(src.reshape(-1))


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1024, 2048])
def test_fp8_struct_path_vs_reference(n, gplk, oracle, cuda):
    import torch
    from gplk import lt

    a = oracle.normal_f32(n * n, n + 41).reshape(n, n)
    b = oracle.normal_f32(n * n, n + 42).reshape(n, n)
    qa, sa = oracle.quantize_fp8(a)
    qb, sb = oracle.quantize_fp8(b)
    tA, tB = torch.from_numpy(qa).to(cuda), torch.from_numpy(qb).to(cuda)
    sc = torch.tensor([sa, sb], dtype=torch.float32, device=cuda)

    g = lt.LtGemm()
    lt.lt_init(g, lt.PREC_FP8, n)
    try:
        assert g.ready and g.n == n and g.prec == lt.PREC_FP8
        _seed(lt.device_view(g.dA, n * n), tA)
        _seed(lt.device_view(g.dB, n * n), tB)
        lt.device_view(g.dScaleA, 1, "<f4").copy_(sc[:1])
        lt.device_view(g.dScaleB, 1, "<f4").copy_(sc[1:])
        torch.cuda.synchronize()
        lt.lt_enqueue(g, 2)  # two GEMMs into the same D: same result
        torch.cuda.synchronize()
        ours = lt.device_view(g.dD, n * n, "<i2").view(torch.bfloat16).float().cpu().numpy().reshape(n, n)
    finally:
        lt.lt_free(g)
    assert not g.ready

    if oracle.ref_available():
        L = oracle.ref_lib()
        r = L.ref_lt_new()
        assert L.gpl_lt_init(r, oracle.PREC["fp8"], n, torch.cuda.current_stream().cuda_stream) == 0
        try:
            ptrs = (ctypes.c_void_p * 7)()
            L.ref_lt_ptrs(r, ptrs)
            dA, dB, _, dD, dSA, dSB, _ = [p for p in ptrs]
            torch.cuda.synchronize()
            _seed(lt.device_view(dA, n * n), tA)
            _seed(lt.device_view(dB, n * n), tB)
            lt.device_view(dSA, 1, "<f4").copy_(sc[:1])
            lt.device_view(dSB, 1, "<f4").copy_(sc[1:])
            torch.cuda.synchronize()
            assert L.gpl_lt_enqueue(r, 1) == 0
            torch.cuda.synchronize()
            ref = lt.device_view(dD, n * n, "<i2").view(torch.bfloat16).float().cpu().numpy().reshape(n, n)
        finally:
            L.gpl_lt_free(r)
            L.ref_lt_delete(r)
        assert _rel_fro(ours, ref) <= TOL

    rng = np.random.default_rng(n)
    pairs = np.stack([rng.integers(0, n, 2048), rng.integers(0, n, 2048)], axis=1)
    want = oracle.gemm_fp8_tn(qa, qb, sa, sb, pairs)
    assert _rel_fro(ours[pairs[:, 1], pairs[:, 0]], want) <= TOL


@pytest.mark.gpu
def test_fp4_struct_path_vs_cublaslt(gplk, oracle, cuda):
    import torch
    from gplk import lt

    n = 2048
    a = oracle.normal_f32(n * n, 7).reshape(n, n)
    b = oracle.normal_f32(n * n, 8).reshape(n, n)
    pa, sfa, ga = oracle.quantize_nvfp4(a)
    pb, sfb, gb = oracle.quantize_nvfp4(b)
    alpha = ga * gb
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda)  # noqa: E731
    tA, tB, tSA, tSB = t(pa), t(pb), t(sfa), t(sfb)

    g = lt.LtGemm()
    lt.lt_init(g, lt.PREC_FP4, n)
    try:
        sfn = gplk.nvfp4_sf_bytes(n, n)
        assert sfn == sfa.size
        _seed(lt.device_view(g.dA, n * n // 2), tA)
        _seed(lt.device_view(g.dB, n * n // 2), tB)
        _seed(lt.device_view(g.dSFA, sfn), tSA)
        _seed(lt.device_view(g.dSFB, sfn), tSB)
        lt.device_view(g.dAlpha, 1, "<f4").fill_(alpha)
        torch.cuda.synchronize()
        lt.lt_enqueue(g, 1)
        torch.cuda.synchronize()
        ours = lt.device_view(g.dD, n * n, "<i2").view(torch.bfloat16).float().cpu().numpy().reshape(n, n)
    finally:
        lt.lt_free(g)

    ref = torch.empty((n, n), dtype=torch.bfloat16, device=cuda)
    ws = torch.empty(32 << 20, dtype=torch.uint8, device=cuda)
    rc = oracle.lt_lib().oracle_lt_gemm_nvfp4_tn(tA.data_ptr(), tB.data_ptr(), tSA.data_ptr(), tSB.data_ptr(),
                                                 ref.data_ptr(), n, n, n, alpha, ws.data_ptr(), ws.numel(),
                                                 torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert _rel_fro(ours, ref.float().cpu().numpy()) <= TOL
    rng = np.random.default_rng(5)
    pairs = np.stack([rng.integers(0, n, 2048), rng.integers(0, n, 2048)], axis=1)
    want = oracle.gemm_nvfp4_tn(pa, pb, sfa, sfb, n, alpha, pairs)
    assert _rel_fro(ours[pairs[:, 1], pairs[:, 0]], want) <= TOL


@pytest.mark.gpu
def test_init_seeds_reference_fill(gplk, cuda):
    """gpl_lt_init seeds A and B with 0x38 and the scales with 1.0, as the
    reference's init does (runner/src/gemm_lt.cu:102-103); enqueue then
    gives K * 1.0 * 1.0 everywhere for FP8."""
    import torch
    from gplk import lt

    n = 512
    g = lt.LtGemm()
    lt.lt_init(g, lt.PREC_FP8, n)
    try:
        assert int(lt.device_view(g.dA, n * n).min()) == 0x38 == int(lt.device_view(g.dB, n * n).max())
        lt.lt_enqueue(g, 1)
        torch.cuda.synchronize()
        d = lt.device_view(g.dD, n * n, "<i2").view(torch.bfloat16).float()
        assert bool((d == float(n)).all())
    finally:
        lt.lt_free(g)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1000, 1001, 136])
def test_fp8_any_n_through_padded_path(n, gplk, oracle, cuda):
    """The reference takes any n (runner/src/gemm_lt.cu:57-161); sizes the
    kernel cannot read directly (K % 16 != 0) run on K-padded copies that
    every enqueue refreshes from the public dA / dB. Checked against the CPU
    oracle over all of D, and against the reference's own gpl_lt path."""
    import torch
    from gplk import lt

    a = oracle.normal_f32(n * n, n + 5).reshape(n, n)
    b = oracle.normal_f32(n * n, n + 6).reshape(n, n)
    qa, sa = oracle.quantize_fp8(a)
    qb, sb = oracle.quantize_fp8(b)
    tA, tB = torch.from_numpy(qa).to(cuda), torch.from_numpy(qb).to(cuda)
    sc = torch.tensor([sa, sb], dtype=torch.float32, device=cuda)
    g = lt.LtGemm()
    lt.lt_init(g, lt.PREC_FP8, n)
    try:
        assert (g.workspace is not None) == (n % 16 != 0)
        _seed(lt.device_view(g.dA, n * n), tA)
        _seed(lt.device_view(g.dB, n * n), tB)
        lt.device_view(g.dScaleA, 1, "<f4").copy_(sc[:1])
        lt.device_view(g.dScaleB, 1, "<f4").copy_(sc[1:])
        lt.lt_enqueue(g, 1)
        torch.cuda.synchronize()
        ours = lt.device_view(g.dD, n * n, "<i2").view(torch.bfloat16).float().cpu().numpy().reshape(n, n)
        # a rewrite of dA between enqueues is seen by the next one
        lt.device_view(g.dA, n * n).zero_()
        lt.lt_enqueue(g, 1)
        torch.cuda.synchronize()
        zero = lt.device_view(g.dD, n * n, "<i2").view(torch.bfloat16).float()
        assert bool((zero == 0).all())
    finally:
        lt.lt_free(g)
    want = oracle.gemm_fp8_tn(qa, qb, sa, sb)
    assert _rel_fro(ours, want) <= TOL
    if oracle.ref_available():
        L = oracle.ref_lib()
        r = L.ref_lt_new()
        if L.gpl_lt_init(r, oracle.PREC["fp8"], n, torch.cuda.current_stream().cuda_stream) != 0:
            # cuBLASLt finds no FP8 algorithm for this n (odd leading
            # dimensions): the reference cannot run it at all.
            L.ref_lt_delete(r)
            assert n % 16 != 0
            return
        try:
            ptrs = (ctypes.c_void_p * 7)()
            L.ref_lt_ptrs(r, ptrs)
            torch.cuda.synchronize()
            _seed(lt.device_view(ptrs[0], n * n), tA)
            _seed(lt.device_view(ptrs[1], n * n), tB)
            lt.device_view(ptrs[4], 1, "<f4").copy_(sc[:1])
            lt.device_view(ptrs[5], 1, "<f4").copy_(sc[1:])
            torch.cuda.synchronize()
            rc = L.gpl_lt_enqueue(r, 1)
            torch.cuda.synchronize()
            if rc == 0:
                ref = lt.device_view(ptrs[3], n * n, "<i2").view(torch.bfloat16).float().cpu().numpy()
                assert _rel_fro(ours, ref.reshape(n, n)) <= TOL
        finally:
            L.gpl_lt_free(r)
            L.ref_lt_delete(r)


@pytest.mark.gpu
def test_fp4_padded_k_and_rejected_size(gplk, oracle, cuda):
    """NVFP4 at n = 2080 (a multiple of 32, not of 256) through the padded
    path, against the CPU oracle on sampled entries; n = 1000 (rows not on
    16-byte boundaries) is refused with -1."""
    import torch
    from gplk import lt

    g = lt.LtGemm()
    with pytest.raises(gplk.GplkError):
        lt.lt_init(g, lt.PREC_FP4, 1000)
    n = 2080
    a = oracle.normal_f32(n * n, 17).reshape(n, n)
    b = oracle.normal_f32(n * n, 18).reshape(n, n)
    pa, sfa, ga = oracle.quantize_nvfp4(a)
    pb, sfb, gb = oracle.quantize_nvfp4(b)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(cuda)  # noqa: E731
    g = lt.LtGemm()
    lt.lt_init(g, lt.PREC_FP4, n)
    try:
        assert g.workspace is not None
        sfn = gplk.nvfp4_sf_bytes(n, n)
        _seed(lt.device_view(g.dA, n * n // 2), t(pa))
        _seed(lt.device_view(g.dB, n * n // 2), t(pb))
        _seed(lt.device_view(g.dSFA, sfn), t(sfa))
        _seed(lt.device_view(g.dSFB, sfn), t(sfb))
        lt.device_view(g.dAlpha, 1, "<f4").fill_(ga * gb)
        lt.lt_enqueue(g, 1)
        torch.cuda.synchronize()
        ours = lt.device_view(g.dD, n * n, "<i2").view(torch.bfloat16).float().cpu().numpy().reshape(n, n)
    finally:
        lt.lt_free(g)
    rng = np.random.default_rng(9)
    pairs = np.stack([rng.integers(0, n, 4096), rng.integers(0, n, 4096)], axis=1)
    want = oracle.gemm_nvfp4_tn(pa, pb, sfa, sfb, n, ga * gb, pairs)
    assert _rel_fro(ours[pairs[:, 1], pairs[:, 0]], want) <= TOL
