"""memstream triad/copy on the GPU, bit-exact against the oracle (fmaf) and
against the reference's own stream_triad_kernel (oracle/_ref)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

S = 3.0  # triad scalar of the measured configuration


def _dev(x, cuda):
    import torch

    return torch.from_numpy(x).to(cuda)


def _bits(t):
    return t.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("bulk", [False, True], ids=["vec4", "bulk"])
@pytest.mark.parametrize("n", [1, 3, 4, 5, 4099, 8192, 65543, 1 << 20, (1 << 22) + 13])
def test_triad_bitexact(n, bulk, gplk, oracle, cuda):
    import torch

    b = oracle.uniform_f32(n, seed=1)
    c = oracle.uniform_f32(n, seed=2)
    want = oracle.triad_f32(b, c, S)
    a = torch.full((n,), float("nan"), device=cuda)
    gplk.triad(a, _dev(b, cuda), _dev(c, cuda), S, bulk=bulk)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(a), want.view(np.uint32))


def test_triad_empty_is_noop(gplk, cuda):
    import torch

    a = torch.empty(0, device=cuda)
    gplk.triad(a, a, a, S)
    gplk.triad(a, a, a, S, bulk=True)
    torch.cuda.synchronize()


def test_triad_misaligned_operands_take_scalar_path(gplk, oracle, cuda):
    import torch

    n = 10_001
    b = oracle.uniform_f32(n + 1, seed=3)
    c = oracle.uniform_f32(n + 2, seed=4)
    tb, tc = _dev(b, cuda), _dev(c, cuda)
    a = torch.zeros(n + 3, device=cuda)
    gplk.triad(a[3:], tb[1:], tc[2:], S)  # 4-, 8-, 12-byte offsets
    torch.cuda.synchronize()
    want = oracle.triad_f32(np.ascontiguousarray(b[1:]), np.ascontiguousarray(c[2:n + 2]), S)
    assert np.array_equal(_bits(a[3:]), want.view(np.uint32))
    with pytest.raises(gplk.GplkError):
        gplk.triad(a[3:], tb[1:], tc[2:], S, bulk=True)  # bulk copies need 16-byte alignment


def test_triad_other_scalars(gplk, oracle, cuda):
    import torch

    n = 1 << 16
    b = oracle.uniform_f32(n, seed=5, lo=-1e3, hi=1e3)
    c = oracle.uniform_f32(n, seed=6, lo=-1e-3, hi=1e-3)
    for s in (0.5, -2.75, 1e30, 0.0):
        a = torch.empty(n, device=cuda)
        gplk.triad(a, _dev(b, cuda), _dev(c, cuda), s)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(a), oracle.triad_f32(b, c, s).view(np.uint32)), s


def test_copy_exact(gplk, oracle, cuda):
    import torch

    for n in (7, 4096, (1 << 20) + 3):
        src = _dev(oracle.uniform_f32(n, seed=9), cuda)
        dst = torch.empty(n, device=cuda)
        gplk.copy(dst, src)
        torch.cuda.synchronize()
        assert torch.equal(dst, src)


def test_triad_full_size_2p30(gplk, oracle, cuda):
    """The measured configuration: three 2^30-element arrays (4 GiB each),
    b, c ~ U[0,1) seeded, s = 3.0; every element bit-exact."""
    import torch

    n = 1 << 30
    b = oracle.uniform_f32(n, seed=101)
    c = oracle.uniform_f32(n, seed=202)
    tb, tc = _dev(b, cuda), _dev(c, cuda)
    a = torch.empty(n, device=cuda)
    for bulk in (False, True):
        a.fill_(float("nan"))
        gplk.triad(a, tb, tc, S, bulk=bulk)
        torch.cuda.synchronize()
        got = a.cpu().numpy()
        want = np.empty_like(b)
        oracle.triad_into(want, b, c, S)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), bulk


@pytest.mark.skipif(not __import__("oracle").ref_available(), reason="reference not compiled")
def test_triad_matches_reference_kernel(gplk, oracle, cuda):
    """Pin: the reference's stream_triad_kernel (compiled from its source)
    produces the same bits as our kernels and the oracle."""
    import torch

    L = oracle.ref_lib()
    for n in (4099, (1 << 24) + 5):
        b = oracle.uniform_f32(n, seed=11)
        c = oracle.uniform_f32(n, seed=12)
        tb, tc = _dev(b, cuda), _dev(c, cuda)
        ours = torch.empty(n, device=cuda)
        ref = torch.empty(n, device=cuda)
        gplk.triad(ours, tb, tc, S)
        # reference kernel: C = A + scalar * B  ->  C = b + s * c
        rc = L.ref_triad_launch(ref.data_ptr(), tb.data_ptr(), tc.data_ptr(), S, n,
                                torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.equal(ours.view(torch.int32), ref.view(torch.int32))
        assert np.array_equal(_bits(ref), oracle.triad_f32(b, c, S).view(np.uint32))
