"""ctypes front end of the CPU oracle (oracle/gpl_oracle.c) and of the
reference runner compiled from its own sources (oracle/_ref/libgpl_ref.so).

TEST INFRASTRUCTURE ONLY. The parity tests, ``__graft_entry__.smoke()`` and
the CPU-baseline arm of ``bench.py`` use this module as the checker. The
product library (libgplk.so) never imports, links or calls it.

Parity status: the reference ships no golden vectors for its load
generators (its buffers are memset patterns, runner/src/gemm_lt.cu:102-103,
runner/src/workload_memstream.cu:78-79), so the oracle is pinned by running
the reference's own code (libgpl_ref.so: build_role_map, the work
accounting, stream_triad_kernel, the cuBLASLt FP8 wrapper) on the same
seeded inputs, and by the E4M3 tables in tests/golden/.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libgpl_oracle.so"
REF_SO = HERE / "_ref" / "libgpl_ref.so"

_f = ctypes.c_float
_d = ctypes.c_double
_i = ctypes.c_int
_sz = ctypes.c_size_t
_u64 = ctypes.c_uint64
_p = ctypes.c_void_p


def build() -> None:
    """Compile the C oracle (make -C oracle)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            build()
        L = ctypes.CDLL(str(ORACLE_SO))
        L.gplo_splitmix64_at.restype = _u64
        L.gplo_splitmix64_at.argtypes = [_u64, _u64]
        L.gplo_fill_uniform_f32.argtypes = [_p, _sz, _u64, _f, _f]
        L.gplo_fill_normal_f32.argtypes = [_p, _sz, _u64]
        L.gplo_triad_f32.argtypes = [_p, _p, _p, _f, _sz, _i]
        L.gplo_max_threads.restype = _i
        L.gplo_sgemm_f64acc.argtypes = [_p, _p, _p, _i, _i, _i, _i, _i, _i, _i]
        L.gplo_sgemm_f32_naive.argtypes = [_p, _p, _p, _i, _i, _i, _i]
        L.gplo_gemm_nn_f64.argtypes = [_p, _p, _p, _i, _i, _i, _i]
        L.gplo_gemm_nn_i8.argtypes = [_p, _p, _p, _i, _i, _i, _i]
        L.gplo_e4m3_decode.restype = _f
        L.gplo_e4m3_decode.argtypes = [ctypes.c_uint8]
        L.gplo_e4m3_encode.restype = ctypes.c_uint8
        L.gplo_e4m3_encode.argtypes = [_f]
        L.gplo_ue4m3_encode.restype = ctypes.c_uint8
        L.gplo_ue4m3_encode.argtypes = [_f]
        L.gplo_e2m1_decode.restype = _f
        L.gplo_e2m1_decode.argtypes = [ctypes.c_uint8]
        L.gplo_e2m1_encode.restype = ctypes.c_uint8
        L.gplo_e2m1_encode.argtypes = [_f]
        L.gplo_quantize_fp8.restype = _f
        L.gplo_quantize_fp8.argtypes = [_p, _sz, _p]
        L.gplo_sf_offset.restype = _sz
        L.gplo_sf_offset.argtypes = [_i, _i, _i]
        L.gplo_sf_bytes.restype = _sz
        L.gplo_sf_bytes.argtypes = [_i, _i]
        L.gplo_quantize_nvfp4.restype = _f
        L.gplo_quantize_nvfp4.argtypes = [_p, _i, _i, _p, _p]
        L.gplo_bf16_round.restype = _f
        L.gplo_bf16_round.argtypes = [_f]
        L.gplo_gemm_fp8_tn.argtypes = [_p, _p, _i, _i, _i, _f, _f, _p, _sz, _p]
        L.gplo_gemm_nvfp4_tn.argtypes = [_p, _p, _p, _p, _i, _i, _i, _f, _p, _sz, _p]
        L.gplo_fma_chain.restype = _f
        L.gplo_fma_chain.argtypes = [_i, ctypes.c_longlong]
        L.gplo_lcg_chain.restype = ctypes.c_uint32
        L.gplo_lcg_chain.argtypes = [_i, ctypes.c_longlong]
        L.gplo_role_map.argtypes = [_p, _i, _p, _p]
        L.gplo_flops_per_iter.restype = _d
        L.gplo_flops_per_iter.argtypes = [_i, _i]
        L.gplo_bytes_per_iter.restype = _d
        L.gplo_bytes_per_iter.argtypes = [_i, _i]
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


# ------------------------------------------------------------ generators

def uniform_f32(n: int, seed: int, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().gplo_fill_uniform_f32(_ptr(out), n, seed, lo, hi)
    return out


def normal_f32(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().gplo_fill_normal_f32(_ptr(out), n, seed)
    return out


# ------------------------------------------------------------ memstream

def triad_f32(b: np.ndarray, c: np.ndarray, s: float, threads: int = 0) -> np.ndarray:
    """a = fmaf(s, c, b) elementwise (bit-exact reference of the triad)."""
    assert b.dtype == np.float32 and c.dtype == np.float32 and b.shape == c.shape
    a = np.empty_like(b)
    lib().gplo_triad_f32(_ptr(a), _ptr(b), _ptr(c), s, b.size, threads)
    return a


def triad_into(a: np.ndarray, b: np.ndarray, c: np.ndarray, s: float, threads: int = 0) -> None:
    lib().gplo_triad_f32(_ptr(a), _ptr(b), _ptr(c), s, b.size, threads)


def max_threads() -> int:
    return int(lib().gplo_max_threads())


# ------------------------------------------------------------ SGEMM

def sgemm_f64acc(A: np.ndarray, B: np.ndarray, threads: int = 0) -> np.ndarray:
    """Row-major C = A @ B accumulated in double (returns float64)."""
    M, K = A.shape
    K2, N = B.shape
    assert K == K2 and A.dtype == np.float32 and B.dtype == np.float32
    C = np.empty((M, N), dtype=np.float64)
    lib().gplo_sgemm_f64acc(_ptr(A), _ptr(B), _ptr(C), M, N, K, K, N, N, threads)
    return C


def sgemm_f32_naive(A: np.ndarray, B: np.ndarray, threads: int = 0) -> np.ndarray:
    M, K = A.shape
    _, N = B.shape
    C = np.empty((M, N), dtype=np.float32)
    lib().gplo_sgemm_f32_naive(_ptr(A), _ptr(B), _ptr(C), M, N, K, threads)
    return C


def gemm_nn_f64(A: np.ndarray, B: np.ndarray, M: int, N: int, K: int, threads: int = 0) -> np.ndarray:
    """Column-major C = A * B (cublasGemmEx OP_N/OP_N). A: float32 values of
    the M x K matrix stored column-major (numpy shape (K, M)), B: K x N
    column-major (shape (N, K)). Returns C as float64 of shape (N, M)."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    assert A.size == M * K and B.size == K * N
    C = np.empty((N, M), dtype=np.float64)
    lib().gplo_gemm_nn_f64(_ptr(A), _ptr(B), _ptr(C), M, N, K, threads)
    return C


def gemm_nn_i8(A: np.ndarray, B: np.ndarray, M: int, N: int, K: int, threads: int = 0) -> np.ndarray:
    """The same product of S8 matrices, exact, as int32 of shape (N, M)."""
    A = np.ascontiguousarray(A, dtype=np.int8)
    B = np.ascontiguousarray(B, dtype=np.int8)
    assert A.size == M * K and B.size == K * N
    C = np.empty((N, M), dtype=np.int32)
    lib().gplo_gemm_nn_i8(_ptr(A), _ptr(B), _ptr(C), M, N, K, threads)
    return C


def allreduce_bf16_sum(inputs: list) -> np.ndarray:
    """The fabric step's BF16 sum allreduce (ncclAllReduce with ncclSum,
    runner/src/workload_nccl.cu:119-291, on BF16): every rank's buffer (uint16
    BF16 bit patterns) added in FP32 in rank order 0..N-1, rounded once to
    BF16 (RNE). Returns uint16 bit patterns."""
    acc = None
    for x in inputs:
        f = (np.asarray(x, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
        acc = f.copy() if acc is None else (acc + f).astype(np.float32)
    r = bf16_round(acc)
    return (r.view(np.uint32) >> 16).astype(np.uint16)


def f16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 -> IEEE binary16 (RNE) -> float32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


# ------------------------------------------------------------ narrow formats

def e4m3_decode_table() -> np.ndarray:
    return np.array([lib().gplo_e4m3_decode(i) for i in range(256)], dtype=np.float32)


def e4m3_encode(x: float) -> int:
    return int(lib().gplo_e4m3_encode(float(x)))


def e2m1_decode_table() -> np.ndarray:
    return np.array([lib().gplo_e2m1_decode(i) for i in range(16)], dtype=np.float32)


def e2m1_encode(x: float) -> int:
    return int(lib().gplo_e2m1_encode(float(x)))


def quantize_fp8(x: np.ndarray) -> tuple[np.ndarray, float]:
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.empty(x.shape, dtype=np.uint8)
    scale = lib().gplo_quantize_fp8(_ptr(x), x.size, _ptr(q))
    return q, float(scale)


def sf_bytes(rows: int, k: int) -> int:
    return int(lib().gplo_sf_bytes(rows, k))


def sf_offset(r: int, kb: int, k_blocks: int) -> int:
    return int(lib().gplo_sf_offset(r, kb, k_blocks))


def quantize_nvfp4(x: np.ndarray) -> tuple[np.ndarray, np.ndarray, float]:
    """rows x k float32 -> (packed rows x k/2 uint8, scale bytes, global)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    assert k % 16 == 0
    packed = np.empty((rows, k // 2), dtype=np.uint8)
    sf = np.zeros(sf_bytes(rows, k), dtype=np.uint8)
    g = lib().gplo_quantize_nvfp4(_ptr(x), rows, k, _ptr(packed), _ptr(sf))
    return packed, sf, float(g)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 -> bf16 (RNE) -> float32, vectorised in numpy."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def gemm_fp8_tn(A: np.ndarray, B: np.ndarray, scale_a: float, scale_b: float,
                pairs: np.ndarray | None = None) -> np.ndarray:
    """A: M x K E4M3 bytes, B: N x K. Full column-major D (as an (N, M)
    row-major array) or the values at `pairs` ((n_pairs, 2) of (m, n))."""
    M, K = A.shape
    N, K2 = B.shape
    assert K == K2
    if pairs is None:
        out = np.empty((N, M), dtype=np.float64)
        lib().gplo_gemm_fp8_tn(_ptr(A), _ptr(B), M, N, K, scale_a, scale_b, None, 0, _ptr(out))
    else:
        pairs = np.ascontiguousarray(pairs, dtype=np.int64)
        out = np.empty(len(pairs), dtype=np.float64)
        lib().gplo_gemm_fp8_tn(_ptr(A), _ptr(B), M, N, K, scale_a, scale_b, _ptr(pairs),
                               len(pairs), _ptr(out))
    return out


def gemm_nvfp4_tn(A: np.ndarray, B: np.ndarray, SFA: np.ndarray, SFB: np.ndarray, K: int,
                  alpha: float, pairs: np.ndarray | None = None) -> np.ndarray:
    M = A.shape[0]
    N = B.shape[0]
    if pairs is None:
        out = np.empty((N, M), dtype=np.float64)
        lib().gplo_gemm_nvfp4_tn(_ptr(A), _ptr(B), _ptr(SFA), _ptr(SFB), M, N, K, alpha, None, 0,
                                 _ptr(out))
    else:
        pairs = np.ascontiguousarray(pairs, dtype=np.int64)
        out = np.empty(len(pairs), dtype=np.float64)
        lib().gplo_gemm_nvfp4_tn(_ptr(A), _ptr(B), _ptr(SFA), _ptr(SFB), M, N, K, alpha,
                                 _ptr(pairs), len(pairs), _ptr(out))
    return out


# ------------------------------------------------------------ powervirus

def fma_chain(lane: int, steps: int) -> float:
    return float(lib().gplo_fma_chain(lane, steps))


def lcg_chain(lane: int, steps: int) -> int:
    return int(lib().gplo_lcg_chain(lane, steps))


def role_map(weights, slots: int = 64) -> tuple[np.ndarray, np.ndarray]:
    w = np.ascontiguousarray(weights, dtype=np.int32)
    assert w.size == 8
    m = np.zeros(slots, dtype=np.uint8)
    c = np.zeros(8, dtype=np.int32)
    lib().gplo_role_map(_ptr(w), slots, _ptr(m), _ptr(c))
    return m, c


def flops_per_iter(op: int, size: int) -> float:
    return float(lib().gplo_flops_per_iter(op, size))


def bytes_per_iter(op: int, size: int) -> float:
    return float(lib().gplo_bytes_per_iter(op, size))


# ------------------------------------------------------------ the reference itself

_ref = None


def ref_available() -> bool:
    return REF_SO.exists()


def ref_lib() -> ctypes.CDLL:
    """The reference runner's own code (oracle/ref_build.sh)."""
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (oracle/ref_build.sh)")
        L = ctypes.CDLL(str(REF_SO))
        L.ref_triad_launch.restype = _i
        L.ref_triad_launch.argtypes = [_p, _p, _p, _f, _sz, _p]
        L.ref_build_role_map.argtypes = [_p, _i, _p, _p]
        L.ref_flops_per_iter.restype = _d
        L.ref_flops_per_iter.argtypes = [_i, _i, _i]
        L.ref_bytes_per_iter.restype = _d
        L.ref_bytes_per_iter.argtypes = [_i, _i]
        L.ref_powervirus_launch.restype = _i
        L.ref_powervirus_launch.argtypes = [_p, _p, _sz, _i, _p, _i, _sz, _p]
        L.ref_pv_block_dim.restype = _i
        L.gpl_lt_precision_supported.restype = ctypes.c_bool
        L.gpl_lt_precision_supported.argtypes = [_i]
        L.gpl_lt_init.restype = _i
        L.gpl_lt_init.argtypes = [_p, _i, _i, _p]
        L.gpl_lt_enqueue.restype = _i
        L.gpl_lt_enqueue.argtypes = [_p, _i]
        L.gpl_lt_free.restype = None
        L.gpl_lt_free.argtypes = [_p]
        L.ref_lt_new.restype = _p
        L.ref_lt_delete.argtypes = [_p]
        L.ref_lt_ptrs.argtypes = [_p, _p]
        L.ref_gemm_ex.restype = _i
        L.ref_gemm_ex.argtypes = [_i, _p, _p, _p, _i, _p]
        L.ref_ts_new.restype = _p
        L.ref_ts_new.argtypes = [_i, _i]
        L.ref_ts_ptrs.argtypes = [_p, _p]
        L.ref_ts_enqueue.argtypes = [_p, _i]
        L.ref_ts_delete.argtypes = [_p]
        _ref = L
    return _ref


def ref_role_map(weights, tensor_cublas: bool = False) -> tuple[np.ndarray, np.ndarray]:
    w = np.ascontiguousarray(weights, dtype=np.int32)
    m = np.zeros(64, dtype=np.uint8)
    c = np.zeros(8, dtype=np.int32)
    ref_lib().ref_build_role_map(_ptr(w), int(tensor_cublas), _ptr(m), _ptr(c))
    return m, c


# Precision codes of the reference's gpl_prec_t (runner/src/args.h:31-40).
PREC = {"fp32": 1, "tf32": 2, "fp16": 3, "bf16": 4, "fp8": 5, "fp64": 6, "int8": 7, "fp4": 8}
OP = {"sgemm": 1, "fft": 2, "memstream": 3, "powervirus": 4, "observe": 5, "nccl": 6}


# ------------------------------------------------------------ cuBLASLt NVFP4 harness

LT_SO = HERE / "liboracle_lt.so"
_lt = None


def lt_lib() -> ctypes.CDLL:
    """cuBLASLt NVFP4 GEMM with VEC16_UE4M3 block scales (oracle/lt_nvfp4.cu)."""
    global _lt
    if _lt is None:
        if not LT_SO.exists():
            build()
        L = ctypes.CDLL(str(LT_SO))
        L.oracle_lt_gemm_nvfp4_tn.restype = _i
        L.oracle_lt_gemm_nvfp4_tn.argtypes = [_p, _p, _p, _p, _p, _i, _i, _i, _f, _p, _sz, _p]
        L.oracle_lt_gemm_nvfp4_tn_timed.restype = _i
        L.oracle_lt_gemm_nvfp4_tn_timed.argtypes = [_p, _p, _p, _p, _p, _i, _i, _i, _f, _p, _sz, _i, _p,
                                                    ctypes.POINTER(_f)]
        _lt = L
    return _lt
