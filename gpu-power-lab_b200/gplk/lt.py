"""Python view of the runner's held-open GEMM handle (include/gemm_lt.h),
libgplk's drop-in for runner/src/gemm_lt.h:17-43.

    g = LtGemm()
    lt_init(g, PREC_FP8, 1024)        # allocates and seeds A, B, scales
    device_view(g.dA, n * n)          # seed operands through the public fields
    lt_enqueue(g, 1)                  # D = sA * sB * A^T B on g.stream
    device_view(g.dD, n * n, "<i2")   # read the column-major BF16 result
    lt_free(g)

lt_init / lt_enqueue raise on the -1 the C calls return (the C calls log
the reason on stderr).
"""
from __future__ import annotations

import ctypes

import gplk

_p = ctypes.c_void_p

# gpl_prec_t values (runner/src/args.h:31-40).
PREC_FP8 = 5
PREC_FP4 = 8


class LtGemm(ctypes.Structure):
    """gpl_lt_gemm_t, field for field (include/gemm_lt.h)."""

    _fields_ = [
        ("dA", _p), ("dB", _p), ("dC", _p), ("dD", _p),
        ("dScaleA", _p), ("dScaleB", _p), ("dScaleD", _p),
        ("dSFA", _p), ("dSFB", _p), ("dAlpha", _p),
        ("workspace", _p), ("workspace_bytes", ctypes.c_size_t),
        ("stream", _p), ("n", ctypes.c_int), ("prec", ctypes.c_int), ("ready", ctypes.c_bool),
    ]


def _bind():
    L = gplk.lib()
    if not getattr(L, "_lt_bound", False):
        L.gpl_lt_precision_supported.restype = ctypes.c_bool
        L.gpl_lt_precision_supported.argtypes = [ctypes.c_int]
        L.gpl_lt_init.restype = ctypes.c_int
        L.gpl_lt_init.argtypes = [ctypes.POINTER(LtGemm), ctypes.c_int, ctypes.c_int, _p]
        L.gpl_lt_enqueue.restype = ctypes.c_int
        L.gpl_lt_enqueue.argtypes = [ctypes.POINTER(LtGemm), ctypes.c_int]
        L.gpl_lt_free.restype = None
        L.gpl_lt_free.argtypes = [ctypes.POINTER(LtGemm)]
        L._lt_bound = True
    return L


def precision_supported(prec: int) -> bool:
    return bool(_bind().gpl_lt_precision_supported(prec))


def lt_init(g: LtGemm, prec: int, n: int, stream=None) -> None:
    if _bind().gpl_lt_init(ctypes.byref(g), prec, n, gplk._stream(stream)) != 0:
        raise gplk.GplkError("gpl_lt_init", 1)


def lt_enqueue(g: LtGemm, count: int = 1) -> None:
    if _bind().gpl_lt_enqueue(ctypes.byref(g), count) != 0:
        raise gplk.GplkError("gpl_lt_enqueue", 2)


def lt_free(g: LtGemm) -> None:
    _bind().gpl_lt_free(ctypes.byref(g))


def device_view(ptr: int, count: int, typestr: str = "|u1"):
    """A torch tensor over `count` elements of device memory at ptr (no copy)."""
    import torch

    class _A:
        __cuda_array_interface__ = {"shape": (count,), "typestr": typestr, "data": (int(ptr), False),
                                    "version": 3, "strides": None}

    return torch.as_tensor(_A(), device="cuda")
