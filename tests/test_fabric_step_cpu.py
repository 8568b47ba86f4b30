"""Host logic of the runner's per-cycle fabric step
(gpu-power-lab_b200/runner/fabric_step.cu), on CPU: the file rendezvous
between runner processes (3 processes, rank order, a rank that never comes),
the cycle count every rank derives, the bus-bandwidth and median helpers, and
the configuration checks that run before any CUDA call."""
from __future__ import annotations

import ctypes
import multiprocessing as mp
import os
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
DROP = REPO / "gpu-power-lab_b200" / "runner"


@pytest.fixture(scope="module")
def step_lib(tmp_path_factory):
    out = tmp_path_factory.mktemp("fabric_step") / "libfabric_step.so"
    cmd = ["/usr/local/cuda/bin/nvcc", "-shared", "-Xcompiler", "-fPIC", "-std=c++17", "-O1",
           f"-I{REPO / 'include'}", f"-I{DROP}", str(DROP / "fabric_step.cu"), "-o", str(out),
           f"-L{REPO / 'gpu-power-lab_b200'}", "-lgplk", "-Xlinker", f"-rpath={REPO / 'gpu-power-lab_b200'}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return str(out)


def _bind(path):
    L = ctypes.CDLL(path)
    L.gpl_fabric_rendezvous.restype = ctypes.c_int
    L.gpl_fabric_rendezvous.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_double]
    L.gpl_fabric_cycles.restype = ctypes.c_ulonglong
    L.gpl_fabric_cycles.argtypes = [ctypes.c_double, ctypes.c_double, ctypes.c_double]
    L.gpl_fabric_busbw_gbs.restype = ctypes.c_double
    L.gpl_fabric_busbw_gbs.argtypes = [ctypes.c_size_t, ctypes.c_double, ctypes.c_int]
    L.gpl_fabric_median.restype = ctypes.c_double
    L.gpl_fabric_median.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.c_size_t]
    L.gpl_fabric_step_init.restype = ctypes.c_int
    L.gpl_fabric_step_init.argtypes = [ctypes.POINTER(ctypes.c_char_p)]
    L.gpl_fabric_step_enabled.restype = ctypes.c_int
    return L


def _rank(path, d, rank, world, q):
    L = _bind(path)
    mine = bytes([rank + 1]) * 64
    allb = ctypes.create_string_buffer(64 * world)
    rc = L.gpl_fabric_rendezvous(d.encode(), b"gplk", rank, world, mine, 64, allb, 20.0)
    q.put((rank, rc, allb.raw))


def test_rendezvous_three_processes(step_lib, tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(step_lib, str(tmp_path), r, 3, q)) for r in (2, 0, 1)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=60) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    want = b"".join(bytes([r + 1]) * 64 for r in range(3))
    assert [g[1] for g in got] == [0, 0, 0]
    assert all(g[2] == want for g in got)
    assert not list(tmp_path.glob(".*.tmp"))  # every temporary file was renamed into place


def test_rendezvous_times_out_without_peer(step_lib, tmp_path):
    L = _bind(step_lib)
    allb = ctypes.create_string_buffer(128)
    assert L.gpl_fabric_rendezvous(str(tmp_path).encode(), b"gplk", 0, 2, b"x" * 64, 64, allb, 0.2) == -1
    # a zero-length barrier through the same files
    assert L.gpl_fabric_rendezvous(str(tmp_path).encode(), b"ready", 0, 1, None, 0, None, 0.2) == 0
    # arguments out of range are refused before touching the directory
    assert L.gpl_fabric_rendezvous(str(tmp_path).encode(), b"gplk", 2, 2, b"x" * 64, 64, allb, 0.2) == -1


def test_cycles_busbw_median(step_lib):
    L = _bind(step_lib)
    assert L.gpl_fabric_cycles(2.0, 100.0, 100.0) == 10
    assert L.gpl_fabric_cycles(2.05, 100.0, 100.0) == 10
    assert L.gpl_fabric_cycles(0.05, 100.0, 100.0) == 1
    assert L.gpl_fabric_cycles(1.0, 0.0, 0.0) == 1
    assert abs(L.gpl_fabric_busbw_gbs(256 << 20, 1e-3, 8) - 2 * 7 / 8 * (256 << 20) / 1e-3 / 1e9) < 1e-6
    assert L.gpl_fabric_busbw_gbs(256 << 20, 1e-3, 1) == 0.0
    v = (ctypes.c_double * 5)(5.0, 1.0, 3.0, 4.0, 2.0)
    assert L.gpl_fabric_median(v, 5) == 3.0
    v4 = (ctypes.c_double * 4)(4.0, 1.0, 3.0, 2.0)
    assert L.gpl_fabric_median(v4, 4) == 2.5


def _init(path, env, q):
    os.environ.update(env)
    for k in ("GPL_FABRIC", "GPL_FABRIC_WORLD", "GPL_FABRIC_RANK", "GPL_FABRIC_DIR"):
        if k not in env:
            os.environ.pop(k, None)
    L = _bind(path)
    err = ctypes.c_char_p()
    rc = L.gpl_fabric_step_init(ctypes.byref(err))
    q.put((rc, L.gpl_fabric_step_enabled(), err.value))


@pytest.mark.parametrize("env,rc,msg", [
    ({}, 0, None),
    ({"GPL_FABRIC": "bogus"}, -1, b"GPL_FABRIC must be gplk or nccl"),
    ({"GPL_FABRIC": "gplk", "GPL_FABRIC_WORLD": "2"}, -1, b"missing or invalid"),
    ({"GPL_FABRIC": "gplk", "GPL_FABRIC_WORLD": "9", "GPL_FABRIC_RANK": "0", "GPL_FABRIC_DIR": "/tmp"}, -1,
     b"missing or invalid"),
    ({"GPL_FABRIC": "nccl", "GPL_FABRIC_WORLD": "2", "GPL_FABRIC_RANK": "2", "GPL_FABRIC_DIR": "/tmp"}, -1,
     b"missing or invalid"),
])
def test_init_configuration_checks(step_lib, env, rc, msg):
    """Configuration errors are reported before any CUDA call (these run on a
    machine without a GPU); with GPL_FABRIC unset the step stays off."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_init, args=(step_lib, env, q))
    p.start()
    got = q.get(timeout=60)
    p.join(timeout=30)
    assert got[0] == rc and got[1] == 0
    if msg is None:
        assert got[2] is None
    else:
        assert msg in got[2]
