"""The GEMM entry points inside a CUDA graph: captured once, replayed several
times, each replay must reproduce the eager result bit for bit.

This covers the launch forms the library uses: the tcgen05 GEMMs launch with
programmatic stream serialisation, and gplk_sgemm_f32 at 1024^3 is a
cooperative stream-K launch whose flags carry a launch epoch that a replayed
graph freezes (the owning block clears each flag it consumed, so every
replay starts clean)."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def test_gemms_replay_in_cuda_graph(gplk, cuda):
    import torch

    n = 1024
    g = torch.Generator(device=cuda)
    g.manual_seed(17)
    a8 = torch.randint(0, 256, (n, n), dtype=torch.uint8, device=cuda, generator=g) & 0x77
    b8 = torch.randint(0, 256, (n, n), dtype=torch.uint8, device=cuda, generator=g) & 0x77
    one = torch.ones(1, device=cuda)
    ab = (torch.rand(n, n, device=cuda, generator=g) * 2 - 1).to(torch.bfloat16)
    bb = (torch.rand(n, n, device=cuda, generator=g) * 2 - 1).to(torch.bfloat16)
    af = torch.rand(n, n, device=cuda, generator=g) * 2 - 1
    bf = torch.rand(n, n, device=cuda, generator=g) * 2 - 1

    def run(outs, stream=None):
        gplk.gemm_fp8_tn(a8, b8, outs[0], one, one, stream=stream)
        gplk.gemm_nn("bf16", ab, bb, outs[1], n, n, n, stream=stream)
        gplk.sgemm(af, bf, outs[2], stream=stream)

    def buffers():
        return [torch.full((n, n), float("nan"), dtype=torch.bfloat16, device=cuda),
                torch.full((n, n), float("nan"), dtype=torch.bfloat16, device=cuda),
                torch.full((n, n), float("nan"), device=cuda)]

    eager = buffers()
    gplk.status_read()
    side = torch.cuda.Stream(device=cuda)
    with torch.cuda.stream(side):
        run(eager, stream=side)  # also allocates this stream's stream-K workspace before capture
    torch.cuda.synchronize()

    replayed = buffers()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        run(replayed, stream=side)
    for _ in range(3):
        for t in replayed:
            t.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        for want, got in zip(eager, replayed):
            assert torch.equal(want.view(torch.int16) if want.dtype == torch.bfloat16 else want.view(torch.int32),
                               got.view(torch.int16) if got.dtype == torch.bfloat16 else got.view(torch.int32))
    assert gplk.status_read() == (0, 0)
