"""Powervirus kernel: every role runs to completion with the device status
OK; the FMA and INT32 roles are bit-exact against the host restatements; the
tcgen05 tensor role's TMEM accumulator matches inner * (A x B^T)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _setup(gplk, cuda, weights, inner, blocks=0, mma=None, verify=True, stream_mib=64):
    import torch

    m, counts = gplk.pv_role_map(weights)
    role_map = torch.tensor(m, dtype=torch.uint8, device=cuda)
    buf = torch.full((stream_mib << 18,), 1.0, dtype=torch.float32, device=cuda)
    sink = torch.zeros(1 + 1024, dtype=torch.float32, device=cuda)
    sm = torch.cuda.get_device_properties(cuda).multi_processor_count
    nb = blocks or sm
    threads = gplk.pv_block_threads()
    verify_out = torch.zeros(nb * threads, dtype=torch.int32, device=cuda) if verify else None
    cfg = gplk.PvCfg()
    cfg.role_map = role_map.data_ptr()
    cfg.stream_buf = buf.data_ptr()
    cfg.stream_bytes = buf.numel() * 4
    cfg.sink = sink.data_ptr()
    cfg.verify_out = verify_out.data_ptr() if verify else None
    keep = [role_map, buf, sink, verify_out]
    if mma is not None:
        a, b, out = mma
        cfg.mma_a, cfg.mma_b, cfg.mma_out = a.data_ptr(), b.data_ptr(), out.data_ptr()
        keep += [a, b, out]
    cfg.blocks = blocks
    cfg.inner = inner
    return cfg, m, nb, verify_out, keep


def _warp_roles(m, nb, threads):
    warps = threads // 32
    stride = 64 // warps
    return [[m[(w * stride + (b % stride)) % 64] for w in range(warps)] for b in range(nb)]


def test_role_map_matches_oracle(gplk, oracle):
    rng = np.random.default_rng(1)
    for _ in range(200):
        w = (rng.integers(0, 9, 8) * (rng.random(8) < 0.5)).tolist()
        m, c = gplk.pv_role_map(w)
        om, oc = oracle.role_map(w)
        assert m == om.tolist() and c == oc.tolist(), w


def test_fma_and_int32_roles_bitexact(gplk, oracle, cuda):
    import torch

    inner = 64
    cfg, m, nb, vout, keep = _setup(gplk, cuda, [0, 1, 0, 0, 1, 0, 0, 0], inner)
    gplk.powervirus_launch(cfg)
    torch.cuda.synchronize()
    v = vout.cpu().numpy().view(np.uint32).reshape(nb, -1, 32)
    roles = _warp_roles(m, nb, gplk.pv_block_threads())
    fma = [np.float32(oracle.fma_chain(l, inner * 16)).view(np.uint32) for l in range(32)]
    lcg = [oracle.lcg_chain(l, inner * 16) for l in range(32)]
    seen = set()
    for b in range(nb):
        for w, r in enumerate(roles[b]):
            want = fma if r == 1 else lcg
            assert v[b, w].tolist() == [int(x) for x in want], (b, w, r)
            seen.add(r)
    assert seen == {1, 4}


def test_tensor_role_accumulator(gplk, oracle, cuda):
    import torch

    inner = 8
    a = oracle.normal_f32(128 * 128, 21).reshape(128, 128)
    b = oracle.normal_f32(256 * 128, 22).reshape(256, 128)
    qa, _ = oracle.quantize_fp8(a)
    qb, _ = oracle.quantize_fp8(b)
    ta, tb = torch.from_numpy(qa).to(cuda), torch.from_numpy(qb).to(cuda)
    out = torch.full((128, 256), float("nan"), device=cuda)
    cfg, *_rest = _setup(gplk, cuda, [1, 1, 1, 0, 0, 0, 0, 0], inner, blocks=2, mma=(ta, tb, out))
    gplk.powervirus_launch(cfg)
    torch.cuda.synchronize()
    want = oracle.gemm_fp8_tn(qa, qb, 1.0, 1.0).T * inner  # (128, 256)
    got = out.cpu().numpy().astype(np.float64)
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel <= 1e-6, rel


@pytest.mark.parametrize("weights", [[1, 1, 1, 0, 0, 0, 0, 0], [1, 1, 1, 1, 1, 1, 1, 1], [0, 0, 1, 0, 0, 0, 0, 0],
                                     [0, 0, 0, 1, 0, 1, 1, 1], [5, 1, 1, 1, 0, 0, 0, 0]])
def test_mixes_run_clean(weights, gplk, cuda):
    import torch

    cfg, *_rest = _setup(gplk, cuda, weights, inner=256, verify=False)
    for _ in range(3):
        gplk.powervirus_launch(cfg)
    torch.cuda.synchronize()


def test_small_stream_buffer_stays_in_bounds(gplk, cuda):
    """The smallest accepted streaming buffer (64 KiB) is smaller than the L2
    role's 4 MiB window; the window is clamped to the buffer."""
    import torch

    cfg, *_rest = _setup(gplk, cuda, [0, 0, 1, 0, 0, 0, 1, 0], inner=64, verify=False, stream_mib=1)
    cfg.stream_bytes = 64 << 10
    gplk.powervirus_launch(cfg)
    torch.cuda.synchronize()


def test_ramp_block_counts(gplk, cuda):
    import torch

    for nb in (1, 7, 37, 148):
        cfg, *_rest = _setup(gplk, cuda, [1, 1, 1, 0, 0, 0, 0, 0], inner=64, blocks=nb, verify=False)
        gplk.powervirus_launch(cfg)
    torch.cuda.synchronize()


def test_time_boxed_launch_runs_to_its_budget(gplk, cuda):
    """With budget_ns set, every role keeps working until the deadline: a
    launch with a tiny fixed part lasts at least the budget, and stays clean."""
    import torch

    cfg, *_rest = _setup(gplk, cuda, [1, 1, 1, 1, 1, 1, 1, 1], inner=8, verify=False)
    cfg.budget_ns = 3_000_000
    gplk.powervirus_launch(cfg)  # warm-up
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    gplk.powervirus_launch(cfg)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    assert 2.9 <= ms <= 50.0, ms
