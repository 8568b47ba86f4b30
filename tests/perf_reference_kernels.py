"""Times the reference's own GPU paths next to libgplk on the same box and
prints one JSON object (not collected by pytest; run on a GPU):

    python tests/perf_reference_kernels.py

  memstream  stream_triad_kernel compiled from the reference source
             (runner/src/workload_memstream.cu:43-54, its launch geometry)
             vs gplk_triad_f32 / gplk_triad_f32_bulk, 3 x 2^30 FP32
  sgemm      the reference's cublasGemmEx FP32 rung call (COMPUTE_32F,
             oracle/ref_gemm_shim.c) vs gplk_sgemm_f32, 1024 / 2048 / 4096
  fp8        the reference's gemm_lt.cu cuBLASLt FP8 (gpl_lt_enqueue)
             vs gplk_gemm_fp8_tn, 8192^3
  nvfp4      cuBLASLt NVFP4 with VEC16_UE4M3 scales (oracle/lt_nvfp4.cu)
             vs gplk_gemm_nvfp4_tn, 2048..16384
  nn         the reference's cublasGemmEx GEMM rung compiled from
             runner/src/workload_gemm.c (oracle/ref_gemm_shim.c) vs
             gplk_gemm_{bf16,f16,tf32,i8}_nn, 8192^3, identical operands:
             random values and the rung's own 0x3c byte fill
  ladder     FP8 (the reference's gemm_lt.cu) and BF16 (its cublasGemmEx
             call) against libgplk at 1024 / 2048 / 4096, random operands
  nn_ref_calls  four reference cublasGemmEx calls each for BF16 and TF32 at
             8192^3 on random operands and nothing else timed: the launch
             list to put under ncu for the library kernels' DRAM traffic
"""
from __future__ import annotations

import ctypes
import json
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
sys.path[:0] = [str(REPO / "gpu-power-lab_b200"), str(REPO / "oracle")]

import torch  # noqa: E402

import gplk  # noqa: E402
import oracle  # noqa: E402


class Sampler:
    """NVML SM clock and power every 20 ms while a case runs."""

    def __init__(self):
        import threading

        import pynvml

        pynvml.nvmlInit()
        self.nv = pynvml
        self.h = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
        self.samples = []
        self.stop_ev = threading.Event()
        self.thr = threading.Thread(target=self.run, daemon=True)

    def run(self):
        while not self.stop_ev.is_set():
            self.samples.append((self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM),
                                 self.nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0))
            self.stop_ev.wait(0.02)

    def __enter__(self):
        self.thr.start()
        return self

    def __exit__(self, *exc):
        self.stop_ev.set()
        self.thr.join()

    def median(self):
        if not self.samples:
            return None, None
        c = sorted(x[0] for x in self.samples)
        p = sorted(x[1] for x in self.samples)
        return c[len(c) // 2], round(p[len(p) // 2], 1)


def sustained(fn, seconds=1.0, warm_s=0.3):
    """Time fn over about `seconds` after `warm_s` of warm-up; returns
    (ms per call, median SM MHz, median W) for the timed window."""
    s = torch.cuda.current_stream()
    t0 = time.perf_counter()
    calls = 0
    while time.perf_counter() - t0 < warm_s or calls < 3:
        fn()
        calls += 1
        if calls % 16 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    per = max(1, int(calls / max(time.perf_counter() - t0, 1e-3) * 0.05))  # ~50 ms batches
    with Sampler() as smp:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        n = 0
        t1 = time.perf_counter()
        while time.perf_counter() - t1 < seconds:
            for _ in range(per):
                fn()
            n += per
            torch.cuda.synchronize()
        e1.record(s)
        torch.cuda.synchronize()
    mhz, watts = smp.median()
    return e0.elapsed_time(e1) / n, mhz, watts


def timed(fn, reps, warm=3):
    s = torch.cuda.current_stream()
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(reps):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps  # ms


def memstream(out):
    n = 1 << 30
    b = torch.rand(n, device="cuda")
    c = torch.rand(n, device="cuda")
    a = torch.empty(n, device="cuda")
    L = oracle.ref_lib()
    st = torch.cuda.current_stream().cuda_stream
    gb = lambda ms: 12 * n / (ms / 1e3) / 1e9
    out["memstream_GBps"] = {
        "reference_stream_triad_kernel": gb(sustained(lambda: L.ref_triad_launch(a.data_ptr(), b.data_ptr(), c.data_ptr(), 3.0, n, st))[0]),
        "gplk_triad_vec4": gb(sustained(lambda: gplk.triad(a, b, c, 3.0))[0]),
        "gplk_triad_bulk": gb(sustained(lambda: gplk.triad(a, b, c, 3.0, bulk=True))[0]),
        "gplk_copy": 8 * n / (sustained(lambda: gplk.copy(a, b))[0] / 1e3) / 1e9,
        "torch_copy": 8 * n / (sustained(lambda: a.copy_(b))[0] / 1e3) / 1e9,
    }
    del a, b, c


def sgemm(out):
    """The reference rung's cublasGemmEx FP32 call (oracle/ref_gemm_shim.c)
    against gplk_sgemm_f32 at 1024 (the parity case), 2048 (ragged waves of
    128 x 128 tiles: stream-K) and 4096 (the rung's default --size)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    L = oracle.ref_lib()
    st = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    res = {}
    for n in (1024, 2048, 4096):
        A = torch.rand(n, n, device="cuda") * 2 - 1
        B = torch.rand(n, n, device="cuda") * 2 - 1
        C = torch.empty(n, n, device="cuda")
        R = torch.empty(n, n, device="cuda")
        tf = lambda ms: round(2 * n ** 3 / (ms / 1e3) / 1e12, 2)
        case = {}
        for name, fn in (("reference_cublasGemmEx_fp32",
                          lambda: L.ref_gemm_ex(1, A.data_ptr(), B.data_ptr(), R.data_ptr(), n, st())),
                         ("gplk_sgemm", lambda: gplk.sgemm(A, B, C))):
            ms, mhz, w = sustained(fn)
            case[name] = {"tflops": tf(ms), "sm_mhz": mhz, "watts": w}
        res[n] = case
    out["sgemm_TFLOPs"] = res


def fp8(out):
    """Both paths on identical operands: random E4M3 bytes (NaN codes
    excluded) and the reference's own constant 0x38 fill (1.0). Operand
    values change the power draw and with it the clock, so the comparison
    is only fair on the same bytes."""
    n = 8192
    L = oracle.ref_lib()
    g = L.ref_lt_new()
    st = torch.cuda.current_stream().cuda_stream
    assert L.gpl_lt_init(g, oracle.PREC["fp8"], n, st) == 0
    ptrs = (ctypes.c_void_p * 7)()
    L.ref_lt_ptrs(g, ptrs)
    cudart = ctypes.CDLL("libcudart.so.12")
    cudart.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    D = torch.empty(n, n, dtype=torch.bfloat16, device="cuda")
    s = torch.ones(1, device="cuda")
    tf = lambda ms: 2 * n ** 3 / (ms / 1e3) / 1e12
    res = {}
    for label in ("random", "const_0x38"):
        if label == "random":
            A = torch.randint(0, 0x7E, (n, n), dtype=torch.uint8, device="cuda")
            B = torch.randint(0, 0x7E, (n, n), dtype=torch.uint8, device="cuda")
            sign = torch.randint(0, 2, (n, n), dtype=torch.uint8, device="cuda") * 0x80
            A |= sign
            B |= sign.flip(0)
        else:
            A = torch.full((n, n), 0x38, dtype=torch.uint8, device="cuda")
            B = torch.full((n, n), 0x38, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        assert cudart.cudaMemcpy(ptrs[0], A.data_ptr(), n * n, 3) == 0
        assert cudart.cudaMemcpy(ptrs[1], B.data_ptr(), n * n, 3) == 0
        torch.cuda.synchronize()
        r = {}
        for name, fn in (("reference_gemm_lt_cublaslt", lambda: L.gpl_lt_enqueue(g, 1)),
                         ("gplk_gemm_fp8_tn", lambda: gplk.gemm_fp8_tn(A, B, D, s, s)),
                         ("reference_gemm_lt_cublaslt_again", lambda: L.gpl_lt_enqueue(g, 1))):
            ms, mhz, w = sustained(fn)
            r[name] = {"tflops": round(tf(ms), 1), "sm_mhz": mhz, "watts": w}
        res[label] = r
    out["fp8_8192_TFLOPs"] = res
    L.gpl_lt_free(g)
    L.ref_lt_delete(g)


def ladder(out):
    """Smaller rungs of the FP8 and BF16 ladders (--size 1024 / 2048 / 4096),
    random operands, back-to-back launches: the reference's gemm_lt.cu FP8
    path and its cublasGemmEx BF16 call against libgplk."""
    L = oracle.ref_lib()
    cudart = ctypes.CDLL("libcudart.so.12")
    cudart.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    st = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    res = {}
    for n in (1024, 2048, 4096):
        tf = lambda ms: round(2 * n ** 3 / (ms / 1e3) / 1e12, 1)
        g = L.ref_lt_new()
        assert L.gpl_lt_init(g, oracle.PREC["fp8"], n, torch.cuda.current_stream().cuda_stream) == 0
        ptrs = (ctypes.c_void_p * 7)()
        L.ref_lt_ptrs(g, ptrs)
        A = torch.randint(0, 0x7E, (n, n), dtype=torch.uint8, device="cuda")
        B = torch.randint(0, 0x7E, (n, n), dtype=torch.uint8, device="cuda")
        D = torch.empty(n, n, dtype=torch.bfloat16, device="cuda")
        s1 = torch.ones(1, device="cuda")
        torch.cuda.synchronize()
        assert cudart.cudaMemcpy(ptrs[0], A.data_ptr(), n * n, 3) == 0
        assert cudart.cudaMemcpy(ptrs[1], B.data_ptr(), n * n, 3) == 0
        torch.cuda.synchronize()
        case = {}
        for name, fn in (("fp8_reference_gemm_lt_cublaslt", lambda: L.gpl_lt_enqueue(g, 1)),
                         ("fp8_gplk_gemm_fp8_tn", lambda: gplk.gemm_fp8_tn(A, B, D, s1, s1))):
            ms, mhz, w = sustained(fn)
            case[name] = {"tflops": tf(ms), "sm_mhz": mhz, "watts": w}
        L.gpl_lt_free(g)
        L.ref_lt_delete(g)
        Ab = (torch.rand(n, n, device="cuda") * 2 - 1).to(torch.bfloat16)
        Bb = (torch.rand(n, n, device="cuda") * 2 - 1).to(torch.bfloat16)
        Db = torch.empty(n, n, dtype=torch.bfloat16, device="cuda")
        for name, fn in (("bf16_reference_cublasGemmEx",
                          lambda: L.ref_gemm_ex(4, Ab.data_ptr(), Bb.data_ptr(), Db.data_ptr(), n, st())),
                         ("bf16_gplk_gemm_bf16_nn", lambda: gplk.gemm_nn("bf16", Ab, Bb, Db, n, n, n))):
            ms, mhz, w = sustained(fn)
            case[name] = {"tflops": tf(ms), "sm_mhz": mhz, "watts": w}
        res[n] = case
        del A, B, D, Ab, Bb, Db
        torch.cuda.empty_cache()
    out["ladder_TFLOPs"] = res


def nvfp4(out):
    """Identical random packed operands and 0x38 (1.0) block scales for both."""
    res = {}
    for n in (2048, 4096, 8192, 16384):
        A = torch.randint(0, 256, (n, n // 2), dtype=torch.uint8, device="cuda")
        B = torch.randint(0, 256, (n, n // 2), dtype=torch.uint8, device="cuda")
        sfb = gplk.nvfp4_sf_bytes(n, n)
        SF = torch.full((sfb,), 0x38, dtype=torch.uint8, device="cuda")
        D = torch.empty(n, n, dtype=torch.bfloat16, device="cuda")
        al = torch.ones(1, device="cuda")
        ws = torch.empty(32 << 20, dtype=torch.uint8, device="cuda")
        tf = lambda m: 2 * n ** 3 / (m / 1e3) / 1e12
        ms_ours, mhz_o, w_o = sustained(lambda: gplk.gemm_nvfp4_tn(A, B, SF, SF, D, n, al))
        reps = max(5, int(1000.0 / ms_ours))  # about one second
        ms = ctypes.c_float(0)
        with Sampler() as smp:
            rc = oracle.lt_lib().oracle_lt_gemm_nvfp4_tn_timed(
                A.data_ptr(), B.data_ptr(), SF.data_ptr(), SF.data_ptr(), D.data_ptr(), n, n, n, 1.0,
                ws.data_ptr(), ws.numel(), reps, torch.cuda.current_stream().cuda_stream, ctypes.byref(ms))
        mhz_l, w_l = smp.median()
        res[n] = {
            "cublaslt_nvfp4": {"tflops": round(tf(ms.value / reps), 1), "sm_mhz": mhz_l, "watts": w_l}
            if rc == 0 else f"rc={rc}",
            "gplk_gemm_nvfp4_tn": {"tflops": round(tf(ms_ours), 1), "sm_mhz": mhz_o, "watts": w_o},
        }
    out["nvfp4_TFLOPs"] = res


def nn(out):
    n = 8192
    L = oracle.ref_lib()
    prec_code = {"tf32": 2, "f16": 3, "bf16": 4, "i8": 7}  # gpl_prec_t (runner/src/args.h:30-39)
    tf = lambda ms: 2 * n ** 3 / (ms / 1e3) / 1e12
    st = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    res = {}
    for prec in ("bf16", "f16", "tf32", "i8"):
        r = {}
        for label in ("random", "fill_0x3c"):
            if prec == "i8":
                A = torch.randint(-128, 128, (n, n), dtype=torch.int8, device="cuda")
                B = torch.randint(-128, 128, (n, n), dtype=torch.int8, device="cuda")
                D = torch.empty(n, n, dtype=torch.int32, device="cuda")
            else:
                dt = {"bf16": torch.bfloat16, "f16": torch.float16, "tf32": torch.float32}[prec]
                A = (torch.rand(n, n, device="cuda") * 2 - 1).to(dt)
                B = (torch.rand(n, n, device="cuda") * 2 - 1).to(dt)
                D = torch.empty(n, n, dtype=dt, device="cuda")
            if label == "fill_0x3c":
                A.view(torch.uint8).fill_(0x3C)
                B.view(torch.uint8).fill_(0x3C)
            Dr = torch.empty_like(D)
            torch.cuda.synchronize()
            rc = L.ref_gemm_ex(prec_code[prec], A.data_ptr(), B.data_ptr(), Dr.data_ptr(), n, st())
            torch.cuda.synchronize()
            case = {}
            for name, fn in (("reference_cublasGemmEx", lambda: L.ref_gemm_ex(prec_code[prec], A.data_ptr(),
                                                                               B.data_ptr(), Dr.data_ptr(), n,
                                                                               st())),
                             (f"gplk_gemm_{prec}_nn", lambda: gplk.gemm_nn(prec, A, B, D, n, n, n))):
                if name.startswith("reference") and rc != 0:
                    case[name] = f"cublas status {rc}"
                    continue
                ms, mhz, w = sustained(fn)
                case[name] = {"tflops": round(tf(ms), 1), "sm_mhz": mhz, "watts": w}
            r[label] = case
            del A, B, D, Dr
            torch.cuda.empty_cache()
        res[prec] = r
    out["nn_8192_TFLOPs"] = res


def nn_ref_calls(out):
    n = 8192
    L = oracle.ref_lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for prec, code, dt in (("bf16", 4, torch.bfloat16), ("tf32", 2, torch.float32)):
        A = (torch.rand(n, n, device="cuda") * 2 - 1).to(dt)
        B = (torch.rand(n, n, device="cuda") * 2 - 1).to(dt)
        D = torch.empty(n, n, dtype=dt, device="cuda")
        torch.cuda.synchronize()
        out[f"nn_ref_calls_{prec}"] = [L.ref_gemm_ex(code, A.data_ptr(), B.data_ptr(), D.data_ptr(), n, st)
                                       for _ in range(4)]
        torch.cuda.synchronize()
        del A, B, D


if __name__ == "__main__":
    which = sys.argv[1:] or ["memstream", "sgemm", "fp8", "nvfp4", "nn"]
    out = {"device": torch.cuda.get_device_name()}
    for w in which:
        globals()[w](out)
        torch.cuda.empty_cache()
    print(json.dumps(out, indent=1, default=float))
