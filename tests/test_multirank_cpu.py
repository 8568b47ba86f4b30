"""Multi-rank host logic on CPU ranks (gloo, world size 2): the bench's
barrier and max-over-ranks timing, and the duty-cycle loop with its
per-cycle allreduce (the fabric step), run in phase on every rank."""
from __future__ import annotations

import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(repo), str(repo / "gpu-power-lab_b200")]
    import torch

    import bench
    from gplk import rung

    d = bench.Dist(world, backend="gloo")
    d.barrier()
    mx = d.max(float(rank + 1) * 1.5)
    tot = d.sum(1.0)
    buf = torch.full((1 << 16,), float(rank + 1))
    launches = []

    def allreduce():
        d.pg.all_reduce(buf)

    log = rung.run_duty_cycles(cycles=4, on_ms=20, off_ms=10, launch=lambda: launches.append(1), sync=lambda: None,
                               allreduce=allreduce, barrier=d.barrier)
    d.close()
    out.put((rank, mx, tot, float(buf[0]), len(log.burst_start), min(log.launches), sum(launches)))


def test_two_cpu_ranks_barrier_max_and_fabric_cycles():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, mx, tot, val, cycles, min_launch, total in res:
        assert mx == 3.0 and tot == 2.0
        # four cycles, each ending with an allreduce of a buffer that starts
        # at (rank + 1): after k rounds every element is 3 * 2^(k-1)
        assert cycles == 4
        assert val == 3.0 * 2 ** 3
        assert min_launch > 0 and total >= 4


def test_busbw_and_windows():
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "gpu-power-lab_b200"))
    from gplk import rung

    assert rung.allreduce_busbw_gbs(256 << 20, 1.0, 1) == 0.0
    assert rung.allreduce_busbw_gbs(1_000_000_000, 1.0, 8) == pytest.approx(1.75)
    samples = [(0.5, 100.0), (1.5, 900.0), (2.5, 200.0), (3.2, 950.0)]
    assert rung.window_power(samples, [(1.0, 2.0), (3.0, 4.0)]) == [900.0, 950.0]


def _stagger_worker(rank: int, world: int, port: int, out):
    os.environ.update({"RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(repo), str(repo / "gpu-power-lab_b200")]
    import bench
    from gplk import rung

    d = bench.Dist(world, backend="gloo")
    on_ms, off_ms = 40.0, 40.0
    off = rung.phase_offset_s(rank, world, on_ms, off_ms, staggered=True)
    log = rung.run_duty_cycles(cycles=3, on_ms=on_ms, off_ms=off_ms, launch=lambda: None, sync=lambda: None,
                               allreduce=None, barrier=d.barrier, start_offset_s=off)
    d.close()
    out.put((rank, off, log.burst_start))


def test_staggered_phases_on_cpu_ranks():
    """Staggered duty cycles: after the shared barrier, rank r of N starts
    r x period / N later, so the two ranks' bursts interleave."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_stagger_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, off0, starts0), (_, off1, starts1) = res
    assert off0 == 0.0 and off1 == pytest.approx(0.04)
    # rank 1's bursts start half a period (40 ms) after rank 0's, within scheduling slack
    lag = [b - a for a, b in zip(starts0, starts1)]
    assert all(0.025 <= x <= 0.075 for x in lag), lag


def test_phase_offsets():
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "gpu-power-lab_b200"))
    from gplk import rung

    assert rung.phase_offset_s(3, 8, 100, 100, staggered=False) == 0.0
    assert [rung.phase_offset_s(r, 4, 100, 100, True) for r in range(4)] == pytest.approx([0, 0.05, 0.1, 0.15])


def test_fused_burst_end_queues_step_behind_last_launch():
    """Fused mode on a fake device: the launch that reaches the end of the
    burst is not waited for, the allreduce follows it directly, and the
    fabric time comes from the supplied timer."""
    from gplk import rung

    t = [0.0]
    events = []

    def clock():
        return t[0]

    def launch():
        events.append("launch")
        t[0] += 0.004  # each launch takes 4 ms of host time to enqueue and run

    def sync():
        events.append("sync")

    def allreduce():
        events.append("allreduce")

    log = rung.run_duty_cycles(cycles=2, on_ms=20, off_ms=0, launch=launch, sync=sync, allreduce=allreduce,
                               clock=clock, sleep=lambda s: None, fused=True, fabric_time=lambda: 0.5e-3)
    for c in range(2):
        # within one cycle: launches separated by syncs, then launch, allreduce, sync
        seq = events[: events.index("allreduce") + 2]
        events[: len(seq)] = []
        assert seq[-3:] == ["launch", "allreduce", "sync"], seq
        assert seq.count("launch") == log.launches[c]
    assert log.fabric_s == [0.5e-3, 0.5e-3]
    assert all(n >= 4 for n in log.launches)
