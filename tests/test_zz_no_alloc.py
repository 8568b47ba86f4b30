"""The powervirus launch that allocates nothing.

gplk_powervirus_launch_noalloc exists for callers that cannot call
cudaMalloc: a load generator running inside another application's process,
where that application's allocator owns the device memory, or a duty-cycled
burst loop that must not let an allocation synchronise the device mid-burst.
It keeps the streaming window and the atomic sink in a static array inside
libgplk instead of caller buffers.

This file is collected last on purpose (test_zz_*): a run that stops at the
first failure has run every other test before it reaches this one.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# Every role except ATOMIC: an atomic role thread's result sums the values
# its atomicAdds returned, which depend on the order other warps got there.
WEIGHTS = [1, 1, 1, 1, 1, 1, 1, 0]
STREAM_BYTES = 16 << 20
INNER = 64


def _tiles(oracle, cuda):
    import torch

    qa, _ = oracle.quantize_fp8(oracle.normal_f32(128 * 128, 31).reshape(128, 128))
    qb, _ = oracle.quantize_fp8(oracle.normal_f32(256 * 128, 32).reshape(256, 128))
    return torch.from_numpy(qa).to(cuda), torch.from_numpy(qb).to(cuda)


def test_noalloc_matches_regular_launch_twice(gplk, oracle, cuda):
    """Two calls in a row of the no-allocation entry point reproduce the
    regular entry point's output, given the regular one a caller buffer of
    the same size and byte pattern (0x3c) and a zeroed sink: bit-exact for
    the per-thread role values, and within the powervirus test tolerance
    (relative Frobenius 1e-6) for the tcgen05 accumulator."""
    import torch

    m, _ = gplk.pv_role_map(WEIGHTS)
    role_map = torch.tensor(m, dtype=torch.uint8, device=cuda)
    sm = torch.cuda.get_device_properties(cuda).multi_processor_count
    nthreads = sm * gplk.pv_block_threads()
    ta, tb = _tiles(oracle, cuda)

    buf = torch.full((STREAM_BYTES,), 0x3C, dtype=torch.uint8, device=cuda)
    sink = torch.zeros(1 + 1024, dtype=torch.float32, device=cuda)
    ref_verify = torch.zeros(nthreads, dtype=torch.int32, device=cuda)
    ref_mma = torch.full((128, 256), float("nan"), device=cuda)
    cfg = gplk.PvCfg()
    cfg.role_map = role_map.data_ptr()
    cfg.stream_buf = buf.data_ptr()
    cfg.stream_bytes = STREAM_BYTES
    cfg.sink = sink.data_ptr()
    cfg.verify_out = ref_verify.data_ptr()
    cfg.mma_a, cfg.mma_b, cfg.mma_out = ta.data_ptr(), tb.data_ptr(), ref_mma.data_ptr()
    cfg.blocks = 0
    cfg.inner = INNER
    gplk.powervirus_launch(cfg)
    torch.cuda.synchronize()
    want_verify = ref_verify.cpu().numpy()
    want_mma = ref_mma.cpu().numpy().astype(np.float64)
    assert np.isfinite(want_mma).all()

    for call in range(2):
        verify = torch.full((nthreads,), -1, dtype=torch.int32, device=cuda)
        mma_out = torch.full((128, 256), float("nan"), device=cuda)
        gplk.powervirus_launch_noalloc(role_map, STREAM_BYTES, INNER, verify_out=verify, mma=(ta, tb, mma_out))
        torch.cuda.synchronize()
        assert np.array_equal(verify.cpu().numpy(), want_verify), f"call {call}: role values differ"
        got = mma_out.cpu().numpy().astype(np.float64)
        rel = np.linalg.norm(got - want_mma) / np.linalg.norm(want_mma)
        assert rel <= 1e-6, f"call {call}: accumulator rel err {rel}"


def test_noalloc_rejects_window_beyond_maximum(gplk, cuda):
    import torch

    m, _ = gplk.pv_role_map(WEIGHTS)
    role_map = torch.tensor(m, dtype=torch.uint8, device=cuda)
    with pytest.raises(gplk.GplkError):
        gplk.powervirus_launch_noalloc(role_map, gplk.PV_NOALLOC_MAX_STREAM_BYTES + 16, INNER)
    # the largest window is accepted
    gplk.powervirus_launch_noalloc(role_map, gplk.PV_NOALLOC_MAX_STREAM_BYTES, INNER)
    torch.cuda.synchronize()
