"""Python host binding of libgplk.so (the C ABI in include/gplk.h).

Thin ctypes wrappers that take CUDA tensors (torch is only the allocator and
stream provider here) and call the sm_100a kernels. There is no fallback:
if libgplk.so is missing or a call returns a non-OK status, these functions
raise.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
LIB_PATH = PKG / "libgplk.so"

STATUS = {
    0: "ok",
    1: "bad argument",
    2: "kernel launch failed",
    3: "device wait timeout",
    4: "unsupported device",
    5: "cuda error",
}

PV_ROLES = ["tensor", "fma", "dram", "sfu", "int32", "smem", "l2", "atomic"]
PV_SLOTS = 64


class GplkError(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn}: {STATUS.get(status, status)} (status {status})")
        self.status = status


_lib = None
_p = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t
_f = ctypes.c_float


class PvCfg(ctypes.Structure):
    """gplk_pv_cfg (include/gplk.h)."""

    _fields_ = [
        ("role_map", _p),
        ("stream_buf", _p),
        ("stream_bytes", _sz),
        ("sink", _p),
        ("verify_out", _p),
        ("mma_a", _p),
        ("mma_b", _p),
        ("mma_out", _p),
        ("blocks", _i),
        ("inner", _i),
        ("budget_ns", ctypes.c_ulonglong),
    ]


def lib() -> ctypes.CDLL:
    """Load libgplk.so (building it first if this checkout has nvcc and no
    library yet). Raises if it cannot be loaded."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        import importlib.util

        spec = importlib.util.spec_from_file_location("gplk_build", PKG / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    L = ctypes.CDLL(str(LIB_PATH))
    L.gplk_status_string.restype = ctypes.c_char_p
    L.gplk_status_string.argtypes = [_i]
    L.gplk_abi_version.restype = _i
    L.gplk_status_read.restype = _i
    L.gplk_status_read.argtypes = [ctypes.POINTER(_i), ctypes.POINTER(_i), _i]
    L.gplk_triad_f32.restype = _i
    L.gplk_triad_f32.argtypes = [_p, _p, _p, _f, _sz, _p]
    L.gplk_triad_f32_bulk.restype = _i
    L.gplk_triad_f32_bulk.argtypes = [_p, _p, _p, _f, _sz, _p]
    L.gplk_copy_f32.restype = _i
    L.gplk_copy_f32.argtypes = [_p, _p, _sz, _p]
    L.gplk_sgemm_f32.restype = _i
    L.gplk_sgemm_f32.argtypes = [_p, _p, _p, _i, _i, _i, _i, _i, _i, _f, _p, _sz, _p]
    L.gplk_sgemm_workspace_bytes.restype = _sz
    L.gplk_sgemm_workspace_bytes.argtypes = [_i, _i, _i]
    L.gplk_gemm_fp8_tn.restype = _i
    L.gplk_gemm_fp8_tn.argtypes = [_p, _p, _p, _i, _i, _i, _p, _p, _p]
    L.gplk_gemm_nvfp4_tn.restype = _i
    L.gplk_gemm_nvfp4_tn.argtypes = [_p, _p, _p, _p, _p, _i, _i, _i, _p, _p]
    for name in ("gplk_gemm_bf16_nn", "gplk_gemm_f16_nn", "gplk_gemm_tf32_nn", "gplk_gemm_i8_nn"):
        for nm in (name, name + "_acc"):
            getattr(L, nm).restype = _i
            getattr(L, nm).argtypes = [_p, _p, _p, _i, _i, _i, _p]
    L.gplk_selftest_wait_timeout.restype = _i
    L.gplk_selftest_wait_timeout.argtypes = [ctypes.c_ulonglong, _p, _p]
    L.gplk_nvfp4_sf_bytes.restype = _sz
    L.gplk_nvfp4_sf_bytes.argtypes = [_i, _i]
    if hasattr(L, "gplk_powervirus_launch"):
        L.gplk_powervirus_launch.restype = _i
        L.gplk_powervirus_launch.argtypes = [ctypes.POINTER(PvCfg), _p]
        L.gplk_pv_build_role_map.restype = None
        L.gplk_pv_build_role_map.argtypes = [_p, _p, _p]
        L.gplk_pv_block_threads.restype = _i
    if hasattr(L, "gplk_powervirus_launch_noalloc"):
        L.gplk_powervirus_launch_noalloc.restype = _i
        L.gplk_powervirus_launch_noalloc.argtypes = [_p, _sz, _i, _i, _p, _p, _p, _p, _p]
    _lib = L
    return L


def _check(fn: str, st: int) -> None:
    if st != 0:
        raise GplkError(fn, st)


def _stream(stream) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t) -> int:
    return t.data_ptr()


def status_read(clear: bool = True) -> tuple[int, int]:
    code, site = _i(0), _i(0)
    _check("gplk_status_read", lib().gplk_status_read(ctypes.byref(code), ctypes.byref(site), int(clear)))
    return code.value, site.value


def selftest_wait_timeout(budget_ns: int, gave_up=None, stream=None) -> None:
    """Launch the watchdog self-test: a wait that can never complete gives up
    after budget_ns and records a device-wait timeout (see include/gplk.h)."""
    _check("gplk_selftest_wait_timeout", lib().gplk_selftest_wait_timeout(
        budget_ns, gave_up.data_ptr() if gave_up is not None else None, _stream(stream)))


# ------------------------------------------------------------ memstream

def triad(a, b, c, s: float, stream=None, bulk: bool = False) -> None:
    """a = b + s * c (FP32, fused multiply-add per element)."""
    n = b.numel()
    assert a.numel() == n and c.numel() == n
    fn = lib().gplk_triad_f32_bulk if bulk else lib().gplk_triad_f32
    _check("gplk_triad_f32" + ("_bulk" if bulk else ""), fn(_ptr(a), _ptr(b), _ptr(c), s, n, _stream(stream)))


def copy(dst, src, stream=None) -> None:
    _check("gplk_copy_f32", lib().gplk_copy_f32(_ptr(dst), _ptr(src), src.numel(), _stream(stream)))


# ------------------------------------------------------------ SGEMM

def sgemm_workspace_bytes(M: int, N: int, K: int) -> int:
    """Bytes of stream-K workspace gplk_sgemm_f32 uses for this shape on the
    current device (0: the shape runs on whole tiles)."""
    return int(lib().gplk_sgemm_workspace_bytes(M, N, K))


_sgemm_ws: dict = {}


def _workspace(nbytes: int, stream):
    """A workspace of at least nbytes for `stream`, kept per (device, stream)
    so GEMMs on one stream share it and GEMMs on different streams never do.
    torch allocates it (the library itself allocates nothing)."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    key = (s.device.index if s.device.index is not None else torch.cuda.current_device(), s.cuda_stream)
    ws = _sgemm_ws.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(nbytes, dtype=torch.uint8, device=s.device)
        _sgemm_ws[key] = ws
    return ws


def sgemm(A, B, C, stream=None, beta: float = 0.0, workspace="auto") -> None:
    """Row-major C = A @ B + beta * C in FP32 (A: M x K, B: K x N, C: M x N).
    workspace: "auto" (a cached per-stream buffer), None (no stream-K), or a
    uint8 CUDA tensor."""
    M, K = A.shape
    K2, N = B.shape
    assert K == K2 and tuple(C.shape) == (M, N)
    if isinstance(workspace, str):
        need = sgemm_workspace_bytes(M, N, K)
        workspace = _workspace(need, stream) if need else None
    wp = workspace.data_ptr() if workspace is not None else None
    wb = workspace.numel() * workspace.element_size() if workspace is not None else 0
    _check("gplk_sgemm_f32", lib().gplk_sgemm_f32(_ptr(A), _ptr(B), _ptr(C), M, N, K, A.stride(0), B.stride(0),
                                                    C.stride(0), float(beta), wp, wb, _stream(stream)))


# ------------------------------------------------------------ narrow GEMMs

def gemm_fp8_tn(A, B, D, scale_a, scale_b, stream=None) -> None:
    """A: (M, K) uint8 E4M3 rows, B: (N, K), D: (N, M) bf16 storage of the
    column-major M x N result. scale_a/scale_b: 1-element float32 tensors."""
    M, K = A.shape
    N, K2 = B.shape
    assert K == K2 and D.numel() == M * N
    _check("gplk_gemm_fp8_tn", lib().gplk_gemm_fp8_tn(_ptr(A), _ptr(B), _ptr(D), M, N, K, _ptr(scale_a),
                                                        _ptr(scale_b), _stream(stream)))


def nvfp4_sf_bytes(rows: int, k: int) -> int:
    return int(lib().gplk_nvfp4_sf_bytes(rows, k))


def gemm_nvfp4_tn(A, B, SFA, SFB, D, K: int, alpha, stream=None) -> None:
    """A: (M, K/2) packed E2M1, B: (N, K/2), SFA/SFB: scale bytes in the
    VEC16_UE4M3 block layout, D: (N, M) bf16 storage of column-major D."""
    M = A.shape[0]
    N = B.shape[0]
    assert A.shape[1] * 2 == K and B.shape[1] * 2 == K and D.numel() == M * N
    _check("gplk_gemm_nvfp4_tn", lib().gplk_gemm_nvfp4_tn(_ptr(A), _ptr(B), _ptr(SFA), _ptr(SFB), _ptr(D),
                                                            M, N, K, _ptr(alpha), _stream(stream)))


# ------------------------------------------------------------ dense tensor-core GEMMs

_NN = {"bf16": "gplk_gemm_bf16_nn", "f16": "gplk_gemm_f16_nn", "tf32": "gplk_gemm_tf32_nn", "i8": "gplk_gemm_i8_nn"}


def gemm_nn(prec: str, A, B, D, M: int, N: int, K: int, stream=None, accumulate: bool = False) -> None:
    """Column-major D = A @ B (cublasGemmEx NN layout), or D = A @ B + D with
    accumulate (beta = 1). A holds M x K with M contiguous, B holds K x N
    with K contiguous, D holds M x N with M contiguous: as torch tensors, A
    is (K, M), B is (N, K) and D is (N, M), all contiguous.
    prec: bf16 | f16 | tf32 | i8."""
    assert A.numel() == M * K and B.numel() == K * N and D.numel() == M * N
    fn = _NN[prec] + ("_acc" if accumulate else "")
    _check(fn, getattr(lib(), fn)(_ptr(A), _ptr(B), _ptr(D), M, N, K, _stream(stream)))


# ------------------------------------------------------------ powervirus

def pv_role_map(weights) -> tuple[list[int], list[int]]:
    w = (_i * 8)(*[int(x) for x in weights])
    m = (ctypes.c_ubyte * PV_SLOTS)()
    c = (_i * 8)()
    lib().gplk_pv_build_role_map(ctypes.addressof(w), ctypes.addressof(m), ctypes.addressof(c))
    return list(m), list(c)


def pv_block_threads() -> int:
    return int(lib().gplk_pv_block_threads())


def powervirus_launch(cfg: PvCfg, stream=None) -> None:
    _check("gplk_powervirus_launch", lib().gplk_powervirus_launch(ctypes.byref(cfg), _stream(stream)))


PV_NOALLOC_MAX_STREAM_BYTES = 32 << 20


def powervirus_launch_noalloc(role_map, stream_bytes: int, inner: int, blocks: int = 0, verify_out=None,
                              mma=None, stream=None) -> None:
    """The powervirus launch that allocates nothing (gplk_powervirus_launch_noalloc):
    for callers that cannot cudaMalloc, such as a load generator running inside
    another application's process whose allocator owns the device memory.
    The streaming window and the atomic sink live in a static array inside
    libgplk (window at most PV_NOALLOC_MAX_STREAM_BYTES). role_map: uint8 CUDA
    tensor of 64 slots; mma: optional (a, b, out) tensors as for PvCfg."""
    a = b = out = None
    if mma is not None:
        a, b, out = mma
    ptr = lambda t: t.data_ptr() if t is not None else None
    _check("gplk_powervirus_launch_noalloc",
           lib().gplk_powervirus_launch_noalloc(ptr(role_map), stream_bytes, blocks, inner, ptr(verify_out),
                                                ptr(a), ptr(b), ptr(out), _stream(stream)))
