"""Duty-cycled powervirus rung with a fabric step, one process per GPU.

The host loop of the reference's powervirus rung (burst for duty_on_ms,
then a genuinely idle gap; runner/src/workload_powervirus.cu:603-647), with
the step the multi-GPU build adds at the end of every cycle: an allreduce of
a BF16 buffer across all ranks (NCCL over NVLink on the GPU box). Every rank
runs the same cycles in phase; the collective is the only exchange.

The loop is written against three callables so that the same code runs
with the real kernel and NCCL, or on CPU ranks (gloo) in the tests:

  launch()      enqueue one kernel launch (asynchronous)
  sync()        wait for this rank's device work
  allreduce()   the cycle's collective (blocking for the cycle's purposes)
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Callable


@dataclass
class CycleLog:
    """Per-cycle wall-clock marks (time.time(), seconds) and counts."""

    burst_start: list = field(default_factory=list)
    burst_end: list = field(default_factory=list)
    fabric_end: list = field(default_factory=list)
    cycle_end: list = field(default_factory=list)
    launches: list = field(default_factory=list)
    fabric_s: list = field(default_factory=list)


def run_duty_cycles(cycles: int, on_ms: float, off_ms: float, launch: Callable[[], None], sync: Callable[[], None],
                    allreduce: Callable[[], None] | None, barrier: Callable[[], None] | None = None,
                    sync_every: int = 8, clock: Callable[[], float] = time.time,
                    sleep: Callable[[float], None] = time.sleep, start_offset_s: float = 0.0,
                    fused: bool = False, fabric_time: Callable[[], float] | None = None) -> CycleLog:
    """Run `cycles` duty cycles: launch kernels back to back for on_ms
    (syncing every `sync_every` launches, as the reference's batches do),
    then the fabric allreduce, then sleep off_ms. `barrier` (optional) aligns
    the ranks once before the first cycle so the cycles run in phase;
    `start_offset_s` then delays this rank's first cycle, which staggers the
    ranks' phases (rank r of N at r x period / N spreads them evenly). With a
    fabric step every cycle the collective re-aligns the ranks, so staggering
    is meaningful without one (allreduce None).

    fused: the burst's last launch is not waited for; the allreduce is
    queued right behind it on the same stream, so the device goes from the
    burst to the fabric step with no host round trip in between (the launch
    reaching the end of the burst is predicted from the previous launch's
    duration). fabric_time() then gives the step's own time (e.g. from CUDA
    events the allreduce recorded), read after the sync; without it the host
    clock brackets the step."""
    log = CycleLog()
    if barrier is not None:
        barrier()
    if start_offset_s > 0:
        sleep(start_offset_s)
    for _ in range(cycles):
        t0 = clock()
        log.burst_start.append(t0)
        n = 0
        last_s = 0.0  # duration of the previous launch (fused mode)
        while (clock() - t0) * 1e3 < on_ms or (fused and allreduce is not None):
            tl = clock()
            launch()
            n += 1
            if fused and allreduce is not None:
                if (tl - t0 + last_s) * 1e3 >= on_ms:
                    break  # this launch ends the burst: the fabric step goes right behind it
                sync()
                last_s = clock() - tl
            elif n % sync_every == 0:
                sync()
        if not (fused and allreduce is not None):
            sync()
        t1 = clock()
        log.burst_end.append(t1)
        log.launches.append(n)
        if allreduce is not None:
            allreduce()
            sync()
        t2 = clock()
        log.fabric_end.append(t2)
        log.fabric_s.append(fabric_time() if (allreduce is not None and fabric_time is not None) else t2 - t1)
        if off_ms > 0:
            sleep(off_ms / 1e3)
        log.cycle_end.append(clock())
    return log


def allreduce_busbw_gbs(nbytes: int, seconds: float, world: int) -> float:
    """NCCL's bus bandwidth convention for allreduce: 2 (N-1)/N x bytes / t
    (runner/src/workload_nccl.cu:106-117)."""
    if seconds <= 0 or world < 1:
        return 0.0
    return 2.0 * (world - 1) / world * nbytes / seconds / 1e9


def phase_offset_s(rank: int, world: int, on_ms: float, off_ms: float, staggered: bool) -> float:
    """Start offset of `rank` for a staggered duty cycle: ranks spread evenly
    over one period; 0 when aligned."""
    if not staggered or world <= 1:
        return 0.0
    return rank * (on_ms + off_ms) / 1e3 / world


def window_power(samples: list[tuple[float, float]], windows: list[tuple[float, float]]) -> list[float]:
    """Power samples (t, W) that fall inside any of the (start, end) windows."""
    out = []
    j = 0
    windows = sorted(windows)
    for t, w in sorted(samples):
        while j < len(windows) and windows[j][1] < t:
            j += 1
        if j < len(windows) and windows[j][0] <= t <= windows[j][1]:
            out.append(w)
    return out
