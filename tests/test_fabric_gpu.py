"""The fabric step (gplk_fabric_*): an in-place BF16 sum allreduce over NVLink
peer memory. One GPU: the single-rank path (its own buffer only) must leave
the data bit-identical. Two or more GPUs: tests/fabric_ranks.py runs one
process per GPU and checks every rank against the oracle (bit-exact) and
against NCCL; skipped when fewer than two GPUs are visible."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent


def test_single_rank_is_identity(gplk, oracle, cuda):
    import torch
    from gplk.fabric import Fabric

    count = 8 * 100003
    fab = Fabric(None, count * 2, rank=0, world=1)
    try:
        x = (torch.randn(count, generator=torch.Generator().manual_seed(3)) * 8).to(torch.bfloat16)
        buf = fab.tensor(count)
        buf.copy_(x.cuda())
        for _ in range(3):  # three epochs
            fab.allreduce_bf16(count)
        torch.cuda.synchronize()
        got = buf.view(torch.int16).cpu().numpy()
        assert np.array_equal(got, x.view(torch.int16).numpy())
        ref = oracle.allreduce_bf16_sum([x.view(torch.int16).numpy().view(np.uint16)])
        assert np.array_equal(got.view(np.uint16), ref)
    finally:
        fab.close()


def test_bad_arguments(gplk, cuda):
    from gplk.fabric import Fabric

    fab = Fabric(None, 4096, rank=0, world=1)
    try:
        with pytest.raises(gplk.GplkError):
            fab.allreduce_bf16(12)  # not a multiple of 8
        with pytest.raises(gplk.GplkError):
            fab.allreduce_bf16(4096)  # larger than the buffer
    finally:
        fab.close()


@pytest.mark.skipif(int(os.environ.get("GPLK_TEST_GPUS", "0") or 0) < 2, reason="needs GPLK_TEST_GPUS >= 2 GPUs")
def test_multi_rank_matches_oracle_and_nccl():
    import torch

    n = min(torch.cuda.device_count(), int(os.environ["GPLK_TEST_GPUS"]))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", "29533", str(REPO / "tests/fabric_ranks.py"),
           "--mode", "check"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(["timeout", "-k", "30", "300", *cmd], capture_output=True, text=True, env=env)
    line = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert res.returncode == 0 and line, res.stdout[-2000:] + res.stderr[-3000:]
    out = json.loads(line[-1])
    assert out["ok"] and out["world"] == n


def test_local_group_single_gpu_f32_identity(gplk, cuda):
    import torch
    from gplk.fabric import local_group

    (f,) = local_group([0], 1 << 20)
    try:
        count = 4 * 60001
        x = torch.randn(count, generator=torch.Generator().manual_seed(5))
        buf = f.tensor(count, torch.float32)
        buf.copy_(x.cuda())
        f.allreduce(count, torch.float32)
        torch.cuda.synchronize()
        assert torch.equal(buf.cpu(), x)
    finally:
        f.close()


def test_local_group_all_gpus_matches_oracle(gplk, oracle):
    """One process driving every visible GPU (skipped with fewer than two):
    FP32 and BF16 sums in rank order, bit-exact against the oracle."""
    import torch
    from gplk.fabric import local_group

    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs in this process")
    n = min(n, 8)
    group = local_group(list(range(n)), 64 << 20)
    try:
        for dtype, count in ((torch.float32, 4 * (n * 100003 + 1)), (torch.bfloat16, 8 * (n * 70001 + 3))):
            xs = [torch.randn(count, generator=torch.Generator().manual_seed(100 + r)).to(dtype) for r in range(n)]
            for f, x in zip(group, xs):
                f.tensor(count, dtype).copy_(x.to(f"cuda:{f.device}"))
            for f in group:
                torch.cuda.synchronize(f.device)
            for f in group:
                f.allreduce(count, dtype)
            for f in group:
                torch.cuda.synchronize(f.device)
            if dtype == torch.float32:
                want = xs[0].numpy().copy()
                for x in xs[1:]:
                    want = (want + x.numpy()).astype(np.float32)
                for f in group:
                    assert np.array_equal(f.tensor(count, dtype).cpu().numpy().view(np.uint32), want.view(np.uint32))
            else:
                want = oracle.allreduce_bf16_sum([x.view(torch.int16).numpy().view(np.uint16) for x in xs])
                for f in group:
                    assert np.array_equal(f.tensor(count, dtype).view(torch.int16).cpu().numpy().view(np.uint16), want)
        code, site = gplk.status_read()
        assert code == 0, (code, hex(site))
    finally:
        for f in group:
            f.close()
