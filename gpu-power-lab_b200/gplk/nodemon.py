"""Python side of the node-level power sampler (include/gplk_nodemon.h,
libgplk_nodemon.so): one NVML sampler thread per GPU of the node in one
process, polled power and instantaneous power plus the driver's buffered
power samples, on one host timebase.

    mon = NodeMonitor([0, 1, 2, 3], hz=100, drain_ms=50)
    ...                                  # run the rung
    mon.stop()
    s = mon.samples()                    # numpy structured array
    w = mon.node_series(source=POLLED, t0=..., bin_s=0.01, max_bins=...)
    mon.close()
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent.parent / "libgplk_nodemon.so"
POLLED, BUFFERED = 0, 1

SAMPLE_DTYPE = np.dtype([("t_s", np.float64), ("power_w", np.float32), ("instant_w", np.float32),
                         ("device", np.int32), ("source", np.int32)])


class _Sample(ctypes.Structure):
    _fields_ = [("t_s", ctypes.c_double), ("power_w", ctypes.c_float), ("instant_w", ctypes.c_float),
                ("device", ctypes.c_int), ("source", ctypes.c_int)]


assert ctypes.sizeof(_Sample) == SAMPLE_DTYPE.itemsize

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} not built (gpu-power-lab_b200/build.py)")
        L = ctypes.CDLL(str(LIB_PATH))
        L.gplk_nodemon_open.restype = ctypes.c_int
        L.gplk_nodemon_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                        ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
        L.gplk_nodemon_stop.restype = ctypes.c_int
        L.gplk_nodemon_stop.argtypes = [ctypes.c_void_p]
        L.gplk_nodemon_count.restype = ctypes.c_size_t
        L.gplk_nodemon_count.argtypes = [ctypes.c_void_p]
        L.gplk_nodemon_read.restype = ctypes.c_size_t
        L.gplk_nodemon_read.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        L.gplk_nodemon_node_series.restype = ctypes.c_size_t
        L.gplk_nodemon_node_series.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_double, ctypes.c_double,
                                               ctypes.c_void_p, ctypes.c_size_t]
        L.gplk_nodemon_close.restype = ctypes.c_int
        L.gplk_nodemon_close.argtypes = [ctypes.c_void_p]
        _lib = L
    return _lib


class NodeMonitorError(RuntimeError):
    pass


class NodeMonitor:
    def __init__(self, devices, hz: int = 100, drain_ms: int = 50, nvml_path: str | None = None):
        devs = (ctypes.c_int * len(devices))(*[int(d) for d in devices])
        h = ctypes.c_void_p()
        rc = lib().gplk_nodemon_open(nvml_path.encode() if nvml_path else None, len(devices), devs, int(hz),
                                     int(drain_ms), ctypes.byref(h))
        if rc != 0:
            raise NodeMonitorError(f"gplk_nodemon_open failed ({rc})")
        self._h = h
        self.devices = list(devices)

    def stop(self) -> None:
        lib().gplk_nodemon_stop(self._h)

    def samples(self) -> np.ndarray:
        n = int(lib().gplk_nodemon_count(self._h))
        out = np.zeros(n, dtype=SAMPLE_DTYPE)
        k = int(lib().gplk_nodemon_read(self._h, out.ctypes.data, n)) if n else 0
        return out[:k]

    def node_series(self, source: int = POLLED, t0: float = 0.0, bin_s: float = 0.01, max_bins: int = 100000):
        w = np.zeros(max_bins, dtype=np.float64)
        k = int(lib().gplk_nodemon_node_series(self._h, int(source), float(t0), float(bin_s), w.ctypes.data,
                                               max_bins))
        return w[:k]

    def close(self) -> None:
        if self._h:
            lib().gplk_nodemon_close(self._h)
            self._h = ctypes.c_void_p()
