"""Benchmark of the gpu-power-lab load generators on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload memstream|sgemm|fp8|nvfp4|powervirus]

Default workload: the memstream STREAM triad a = b + 3.0 * c over three FP32
arrays of 2^30 elements (4 GiB each; b, c ~ U[0,1) seeded). One step = one
triad launch over the whole arrays. Every GPU runs its own replica (the
workload does not shard): value = bytes moved by all ranks / max-over-ranks
device time. Inputs are 12 GiB per step, far above the 126 MB L2, so no L2
flush is needed between steps.

Other rungs (--workload): sgemm (FP32 1024^3), fp8 (E4M3 8192^3), nvfp4
(E2M1 16384^3) report TFLOP/s; powervirus reports sustained watts.

--impl reference times the reference path's CPU implementation on the host
cores (the oracle port of the triad, all threads), rank 0 only.

Prints ONE JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "gpu-power-lab_b200"
sys.path.insert(0, str(PKG))

TRIAD_N = 1 << 30
TRIAD_S = 3.0
TRIAD_BYTES = 12 * TRIAD_N  # read b, read c, write a (runner/src/workload_util.c:43-47)

# dram__bytes_read.sum + dram__bytes_write.sum per launch from one ncu capture
# of each kernel, scaled to the full launch where the capture was smaller.
NCU_TRAFFIC = {
    "memstream_vec4": 12.58e9,  # 8 x 1.573 GB (3 x 2^27 capture)
    "memstream_bulk": 12.58e9,  # 8 x 1.572 GB (3 x 2^27 capture)
    "sgemm": 8.4e6,             # 1024^3
    "fp8": 339.8e6,             # 8192^3 (odd raster groups walking N backwards)
    "nvfp4": 1343.6e6,          # 16384^3
    "bf16": 1149.9e6,           # 8192^3
    "tf32": 2452.5e6,           # 8192^3
}

NOMINAL_TFLOPS = {"fp8": 4500.0, "nvfp4": 9000.0, "sgemm": 148 * 128 * 2 * 1.965e9 / 1e12,
                  "bf16": 2250.0, "f16": 2250.0, "tf32": 1125.0, "i8": 4500.0}
# The dense cublasGemmEx precisions of the ladder (runner/src/workload_gemm.c:44-79), column-major NN.
NN_GEMMS = {"bf16": ("bf16", "BF16 NN GEMM M=N=K=8192, FP32 accumulate, BF16 out"),
            "f16": ("f16", "FP16 NN GEMM M=N=K=8192, FP32 accumulate, FP16 out"),
            "tf32": ("tf32", "TF32 NN GEMM M=N=K=8192, FP32 in/out"),
            "i8": ("s8", "INT8 NN GEMM M=N=K=8192, S32 accumulate and out")}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["memstream", "sgemm", "fp8", "nvfp4", "bf16", "f16", "tf32", "i8",
                                           "powervirus", "fabric"],
                    default="memstream")
    ap.add_argument("--kernel", choices=["vec4", "bulk"], default="bulk",
                    help="memstream kernel variant")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--phase", choices=["aligned", "staggered"], default="aligned",
                    help="powervirus: ranks' duty cycles in phase, or spread evenly over one period "
                         "(staggered drops the per-cycle fabric step, which would re-align them)")
    ap.add_argument("--fabric", choices=["nccl", "gplk"], default="nccl",
                    help="powervirus fabric step: NCCL all_reduce, or gplk_fabric_allreduce_bf16 over NVLink peers")
    ap.add_argument("--fabric-mib", type=int, default=256, help="fabric allreduce size (BF16), MiB")
    ap.add_argument("--gemm-n", type=int, default=0,
                    help="M = N = K of the tensor-core GEMM workloads (0: 8192, 16384 for nvfp4)")
    ap.add_argument("--sgemm-n", type=int, default=1024,
                    help="sgemm workload size M = N = K (1024 is the parity configuration; the rung's --size "
                         "default is 4096)")
    ap.add_argument("--mix", default="4,1,2", help="powervirus role weights tensor,fma,dram[,sfu,int32,smem,l2,atomic]")
    ap.add_argument("--budget-us", type=float, default=1000.0, help="powervirus launch time box")
    ap.add_argument("--duty-on-ms", type=float, default=100.0)
    ap.add_argument("--duty-off-ms", type=float, default=100.0)
    ap.add_argument("--no-rungs", action="store_true",
                    help="memstream at N=1: skip the FP8 / NVFP4 GEMM and power rungs added to the line")
    ap.add_argument("--rung-seconds", type=float, default=1.5,
                    help="sustained run per GEMM rung arm (the power rung runs twice as long)")
    ap.add_argument("--no-pv-cycle", action="store_true",
                    help="memstream at N>1: skip the short in-phase powervirus duty cycle (gplk fabric step per "
                         "cycle) whose node power and fabric time are added to the line")
    ap.add_argument("--no-fabric-check", action="store_true",
                    help="memstream at N>1: skip the fabric step's parity check and timing added to the line")
    ap.add_argument("--elements", type=int, default=TRIAD_N,
                    help="memstream array length (smaller cases are for profiling only)")
    return ap.parse_args()


# ------------------------------------------------------------ distributed plumbing

class Dist:
    """One process per GPU (torchrun env). NCCL on the GPU box; `backend`
    "gloo" runs the same barrier / max-over-ranks logic on CPU ranks."""

    def __init__(self, n_gpus: int, backend: str = "nccl"):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            kw = {}
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                kw["device_id"] = torch.device("cuda", self.local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120), **kw)
            self.pg = dist

    def _dev(self):
        return "cuda" if self.backend == "nccl" else "cpu"

    def barrier(self):
        if self.pg:
            import torch

            t = torch.zeros(1, device=self._dev())
            self.pg.all_reduce(t)
            if self.backend == "nccl":
                torch.cuda.synchronize()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch

        t = torch.tensor([x], dtype=torch.float64, device=self._dev())
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, x: float) -> float:
        if not self.pg:
            return x
        import torch

        t = torch.tensor([x], dtype=torch.float64, device=self._dev())
        self.pg.all_reduce(t)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ------------------------------------------------------------ clocks during the timed region

REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


class ClockSampler:
    """NVML sampling thread: SM clock, throttle reasons and power, every 25 ms."""

    def __init__(self, device_index: int, period_s: float = 0.025):
        self.idx = device_index
        self.period = period_s
        self.samples = []
        self._stop = threading.Event()
        self._thr = None
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_sm = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.limit_w = pynvml.nvmlDeviceGetEnforcedPowerLimit(self.h) / 1000.0
            # Instantaneous power (NVML_FI_DEV_POWER_INSTANT) where the driver
            # has it: the averaged reading smears a 100 ms square wave.
            self.instant_ok = hasattr(pynvml, "NVML_FI_DEV_POWER_INSTANT")
            self.ok = True
        except Exception:
            self.max_sm = None
            self.limit_w = None

    def _sample(self):
        nv = self.nv
        sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
        try:
            reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            reasons = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        power = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0  # driver-averaged
        inst = None
        if self.instant_ok:
            try:
                fv = nv.nvmlDeviceGetFieldValues(self.h, [nv.NVML_FI_DEV_POWER_INSTANT])[0]
                if fv.nvmlReturn == 0:  # milliwatts; the value type varies by driver
                    vt = int(fv.valueType)
                    raw = fv.value.uiVal if vt == 1 else (fv.value.ulVal if vt == 2 else fv.value.ullVal)
                    inst = raw / 1000.0
            except Exception:
                self.instant_ok = False
        self.samples.append((time.time(), sm, reasons, inst if inst is not None else power))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                pass
            self._stop.wait(self.period)

    def start(self):
        if self.ok:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()

    def stop(self):
        if self._thr:
            self._stop.set()
            self._thr.join()
            if not self.samples:
                try:
                    self._sample()
                except Exception:
                    pass

    def power_stats(self, skip_s: float = 0.0) -> dict:
        """Mean and percentiles of the power samples taken more than skip_s
        after the first sample (the controller settles in the first ~0.3 s)."""
        if not self.samples:
            return {"avg_w": None, "samples": 0}
        t0 = self.samples[0][0]
        w = sorted(s[3] for s in self.samples if s[0] - t0 >= skip_s) or sorted(s[3] for s in self.samples)
        pct = lambda q: w[min(len(w) - 1, int(q * (len(w) - 1)))]  # noqa: E731
        return {"avg_w": round(sum(w) / len(w), 1), "p5_w": round(pct(0.05), 1), "p95_w": round(pct(0.95), 1),
                "max_w": round(w[-1], 1), "samples": len(w), "limit_w": self.limit_w}

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_sm, "reasons": [], "samples": 0}
        sms = sorted(s[1] for s in self.samples)
        mask = 0
        for s in self.samples:
            mask |= int(s[2])
        reasons = [name for bit, name in REASONS.items() if mask & bit and bit != 0x1]
        pw = sorted(s[3] for s in self.samples)
        return {
            "sm_mhz": sms[len(sms) // 2],
            "sm_max_mhz": self.max_sm,
            "reasons": reasons,
            "samples": len(self.samples),
            "power_w_median": round(pw[len(pw) // 2], 1),
            "power_limit_w": self.limit_w,
        }


def measured_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["_source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "_source": "fallback"}


# ------------------------------------------------------------ CPU baseline (oracle port)

def host_threads() -> int:
    """Every core this process may run on. Passed to the host loops
    explicitly, so torchrun's OMP_NUM_THREADS=1 does not shrink them."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_triad_gbps(seconds: float, n: int = 1 << 28, threads: int = 0, single: bool = True) -> dict:
    """The host triad a = fmaf(s, c, b) (the oracle's restatement of the
    triad) over n elements, repeated for about `seconds`, all cores; with
    `single`, also one thread for about a fifth of that."""
    sys.path.insert(0, str(REPO / "oracle"))
    import numpy as np
    import oracle

    b = oracle.uniform_f32(n, seed=101)
    c = oracle.uniform_f32(n, seed=202)
    a = np.empty_like(b)
    nthreads = threads or host_threads()
    oracle.triad_into(a, b, c, TRIAD_S, nthreads)  # first touch
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.triad_into(a, b, c, TRIAD_S, nthreads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    out = {"value": round(12 * n * reps / el / 1e9, 2), "unit": "GB/s", "cores": nthreads, "kind": "port",
           "sample": f"{reps} host triads over 3 x 2^{n.bit_length() - 1} FP32 ({el:.1f} s)"}
    if single and nthreads > 1:
        reps1, t1 = 0, time.perf_counter()
        while True:
            oracle.triad_into(a, b, c, TRIAD_S, 1)
            reps1 += 1
            el1 = time.perf_counter() - t1
            if el1 >= seconds / 5:
                break
        out["single_thread_gbps"] = round(12 * n * reps1 / el1 / 1e9, 2)
        out["single_thread_sample"] = f"{reps1} host triads on one thread ({el1:.1f} s)"
    return out


def cpu_sgemm_tflops(n: int, seconds: float) -> dict:
    """The host C11 triple loop (the oracle's gplo_sgemm_f32_naive: row-major,
    FP32 accumulate in k order) on the n^3 problem's operands, all cores with
    OpenMP, and single-threaded on a row slab sized to about a tenth of
    `seconds`. Reported beside the GPU number, not a target."""
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle

    A = oracle.uniform_f32(n * n, seed=0, lo=-1.0, hi=1.0).reshape(n, n)
    B = oracle.uniform_f32(n * n, seed=1, lo=-1.0, hi=1.0).reshape(n, n)
    nthreads = host_threads()
    # Whole problem up to 1024^3; above that a row slab of about 2 GFLOP.
    slab = n if n <= 1024 else max(16, (1 << 30) // (n * n))
    As = A if slab == n else A[:slab].copy()
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.sgemm_f32_naive(As, B, nthreads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    rows = 16
    t1 = time.perf_counter()
    oracle.sgemm_f32_naive(A[:rows].copy(), B, 1)
    one = 2.0 * rows * n * n / (time.perf_counter() - t1) / 1e12
    what = f"{n}^3" if slab == n else f"a {slab}-row slab of the {n}^3 problem"
    return {"value": round(2.0 * slab * n * n * reps / el / 1e12, 4), "unit": "TFLOP/s", "cores": nthreads,
            "kind": "port", "single_thread_tflops": round(one, 5),
            "sample": f"{reps} host triple-loop SGEMMs on {what}, {nthreads} threads ({el:.1f} s); "
                      f"single thread timed on a {rows}-row slab"}


# ------------------------------------------------------------ memstream

def bench_memstream(args, dist: Dist) -> dict:
    import torch
    import gplk

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    gplk.lib()
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + dist.rank)
    n = args.elements
    nbytes = 12 * n
    b = torch.rand(n, device=dev, generator=g)
    c = torch.rand(n, device=dev, generator=g)
    a = torch.empty(n, device=dev)
    stream = torch.cuda.current_stream(dev)
    bulk = args.kernel == "bulk"

    def step():
        gplk.triad(a, b, c, TRIAD_S, stream=stream, bulk=bulk)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(dist.local)
    dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    sampler.stop()
    ms = e0.elapsed_time(e1)
    ms_max = dist.max(ms)
    code, site = gplk.status_read()
    if code != 0:
        raise RuntimeError(f"device status {code} at {site:#x}")

    per_launch_s = ms / 1e3 / args.steps
    achieved = nbytes / per_launch_s / 1e9
    peaks = measured_peaks()
    value = dist.world * nbytes * args.steps / (ms_max / 1e3) / 1e9

    e2e = None
    if not args.no_e2e:
        e2e = memstream_e2e(a, b, c, stream, bulk, dist, steps=3)
    if n != TRIAD_N:
        workload = f"memstream STREAM triad a = b + 3.0*c, FP32, 3 x {n} elements (profiling case)"
    else:
        workload = "memstream STREAM triad a = b + 3.0*c, FP32, 3 x 2^30 elements (4 GiB each)"

    traffic = NCU_TRAFFIC["memstream_bulk" if bulk else "memstream_vec4"] if n == TRIAD_N else None
    out = {
        "metric": "memstream triad GB/s",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": dist.world,
        "steps": args.steps,
        "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: b, c ~ U[0,1) from torch's seeded generator, s = 3.0",
        "config": {"workload": workload,
                   "elements": n, "bytes_per_step_per_gpu": nbytes,
                   "kernel": "triad_bulk" if bulk else "triad_vec4",
                   "l2": "inputs (12 GiB per step) larger than the 126 MB L2; no flush",
                   "parallelism": f"replicas x{dist.world} (the workload does not shard)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                     "peak_source": f"{peaks['_source']} hbm_gbs (burst copy)",
                     "algorithmic_bytes_per_launch": nbytes},
        "clocks": sampler.summary(),
        "gpu_launches": args.steps,
    }
    if e2e:
        out["e2e"] = e2e
    return out


def memstream_e2e(a, b, c, stream, bulk, dist: Dist, steps: int, chunk: int = 1 << 24) -> dict:
    """The same triad through the C ABI with host buffers: every step copies
    b and c from pinned host memory, runs the triad and reads a back, all of
    it. The arrays move in chunks of `chunk` elements on three streams
    (copy in, triad, copy out), so the host-to-device copies of later chunks
    overlap the device-to-host copies of earlier ones: PCIe carries both
    directions at once. Events keep every chunk's order: a chunk is
    overwritten only after the previous step's triad read it, and a is
    rewritten only after the previous step copied it out."""
    import torch
    import gplk

    n = b.numel()
    hb = torch.empty(n, dtype=torch.float32, pin_memory=True)
    hc = torch.empty(n, dtype=torch.float32, pin_memory=True)
    ha = torch.empty(n, dtype=torch.float32, pin_memory=True)
    hb.copy_(b, non_blocking=False)
    hc.copy_(c, non_blocking=False)
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    bounds = [(k, min(k + chunk, n)) for k in range(0, n, chunk)]
    ev_in = [torch.cuda.Event() for _ in bounds]
    ev_tr = [torch.cuda.Event() for _ in bounds]
    ev_out = [torch.cuda.Event() for _ in bounds]
    first = [True]

    def step():
        for i, (lo, hi) in enumerate(bounds):
            if not first[0]:
                s_in.wait_event(ev_tr[i])  # the previous step's triad has read b, c here
            with torch.cuda.stream(s_in):
                b[lo:hi].copy_(hb[lo:hi], non_blocking=True)
                c[lo:hi].copy_(hc[lo:hi], non_blocking=True)
                ev_in[i].record(s_in)
            stream.wait_event(ev_in[i])
            if not first[0]:
                stream.wait_event(ev_out[i])  # the previous step has copied a out of here
            gplk.triad(a[lo:hi], b[lo:hi], c[lo:hi], TRIAD_S, stream=stream, bulk=bulk)
            ev_tr[i].record(stream)
            s_out.wait_event(ev_tr[i])
            with torch.cuda.stream(s_out):
                ha[lo:hi].copy_(a[lo:hi], non_blocking=True)
                ev_out[i].record(s_out)
        first[0] = False

    step()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for _ in range(steps):
        step()
    s_out.wait_event(ev_tr[-1])
    e1.record(s_out)  # after the last copy out, which follows every chunk's triad
    torch.cuda.synchronize()
    ms = dist.max(e0.elapsed_time(e1))
    value = dist.world * 12 * n * steps / (ms / 1e3) / 1e9
    return {"value": round(value, 2), "unit": "GB/s", "h2d_bytes_per_step": 8 * n,
            "d2h_bytes_per_step": 4 * n, "steps": steps,
            "note": f"pinned host b, c -> device, triad, device a -> pinned host, per step, in "
                    f"{len(bounds)} chunks on three streams (copy in / triad / copy out overlap)"}


# ------------------------------------------------------------ GEMM rungs

def bench_gemm(args, dist: Dist) -> dict:
    import torch
    import gplk

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    gplk.lib()
    g = torch.Generator(device=dev)
    g.manual_seed(7 + dist.rank)
    stream = torch.cuda.current_stream(dev)
    w = args.workload
    if w == "sgemm":
        n = args.sgemm_n
        A = torch.rand(n, n, device=dev, generator=g) * 2 - 1
        B = torch.rand(n, n, device=dev, generator=g) * 2 - 1
        C = torch.empty(n, n, device=dev)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

        def step():
            flush.zero_()  # 256 MiB write: evicts the 12 MiB working set from L2
            gplk.sgemm(A, B, C, stream=stream)

        dtype, workload = "f32", f"FP32 SGEMM C = A*B row-major, M=N=K={n}, U[-1,1)"
        launches_per_step = 2

        def sgemm_library():
            # cuBLAS in true FP32 (TF32 off), the library behind the reference
            # rung's cublasGemmEx COMPUTE_32F call.
            torch.backends.cuda.matmul.allow_tf32 = False
            return torch.matmul(A, B)

        case = {"flops": 2.0 * n ** 3, "ours": lambda: gplk.sgemm(A, B, C), "library": sgemm_library,
                "library_name": "cuBLAS FP32 via torch.matmul (TF32 off)", "lib_view": lambda out: out,
                "ours_view": lambda: C, "inputs": [A, B], "D": C}
    else:
        n = args.gemm_n or (16384 if w == "nvfp4" else 8192)
        case = _gemm_case(w, n, dev, stream, seed=31 + 7 * dist.rank)
        step = case["ours"]
        dtype, workload = case["dtype"], case["workload"]
        launches_per_step = 1
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(dist.local)
    dist.barrier()
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    sampler.stop()
    ms = e0.elapsed_time(e1)
    ms_max = dist.max(ms)
    flops = 2.0 * n ** 3
    # Kernel-only duration for the roofline: time the GEMM alone (no flush).
    if w == "sgemm":
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(stream)
        for _ in range(args.steps):
            gplk.sgemm(A, B, C, stream=stream)
        k1.record(stream)
        torch.cuda.synchronize()
        kernel_s = k0.elapsed_time(k1) / 1e3 / args.steps
    else:
        kernel_s = ms / 1e3 / args.steps
    achieved = flops / kernel_s / 1e12
    value = dist.world * flops * args.steps / (ms_max / 1e3) / 1e12
    peak, peak_source = NOMINAL_TFLOPS[w], "nominal dense"
    if w in ("bf16", "f16"):
        # The pool's measured dense BF16 rate (cuBLAS, burst) is the roofline
        # for the 16-bit kinds; the other kinds have no measured figure.
        pk = measured_peaks()
        peak = pk["bf16_tflops"]
        peak_source = f"{pk['_source']} bf16_tflops (burst cuBLAS BF16 8192^3); nominal {NOMINAL_TFLOPS[w]:.0f}"
    scalar_ffma = None
    if w == "sgemm":
        # Scalar FFMA alone stays well below the nominal FP32 rate on B200
        # (paired FFMA2 is what reaches it), so it is context, not the peak.
        peak_source = "nominal: 148 SMs x 128 FP32 lanes x 2 flop x 1965 MHz"
        scalar_ffma = fma_peak_tflops(dev, stream)
    return {
        "metric": f"{w} TFLOP/s", "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": dist.world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic, seeded",
        "config": {"workload": workload, "size": n,
                   "l2": "256 MiB L2 flush per step" if w == "sgemm" else "operands larger than L2",
                   "parallelism": f"replicas x{dist.world}"},
        "roofline": {"bound": "tensor" if w != "sgemm" else "fp32-simt", "achieved": round(achieved, 1),
                     "peak": round(peak, 1), "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "traffic": NCU_TRAFFIC.get(w) if n == {"sgemm": 1024, "nvfp4": 16384}.get(w, 8192) else None,
                     "peak_source": peak_source,
                     **({"scalar_ffma_measured": scalar_ffma} if scalar_ffma is not None else {})},
        "clocks": sampler.summary(),
        "gpu_launches": args.steps * (1 if w != "sgemm" else 1),
        **_sustained_extras(case, stream, dev, args.rung_seconds),
    }


def fma_peak_tflops(dev, stream, inner: int = 10000, launches: int = 60) -> dict:
    """Scalar-FFMA throughput of this GPU, measured: gplk_powervirus_launch
    with every warp slot on the FMA role and fixed work (each thread runs
    eight dependent FFMA chains for inner x 16 steps), one 32-warp block per
    SM, `launches` launches (about a third of a second) timed with CUDA
    events after two warm-up launches, with the SM clock sampled meanwhile."""
    import gplk
    import torch

    role_map, _ = gplk.pv_role_map([0, 1, 0, 0, 0, 0, 0, 0])
    role = torch.tensor(role_map, dtype=torch.uint8, device=dev)
    buf = torch.zeros((64 << 10) // 4, device=dev)
    sink = torch.zeros(1 + 1024, device=dev)
    cfg = gplk.PvCfg(role_map=role.data_ptr(), stream_buf=buf.data_ptr(), stream_bytes=64 << 10,
                     sink=sink.data_ptr(), blocks=0, inner=inner, budget_ns=0)
    for _ in range(2):
        gplk.powervirus_launch(cfg, stream=stream)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(dev.index if dev.index is not None else 0, period_s=0.01)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(launches):
        gplk.powervirus_launch(cfg, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    sampler.stop()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    flops = launches * sms * gplk.pv_block_threads() * 8 * inner * 16 * 2
    tflops = flops / (e0.elapsed_time(e1) / 1e3) / 1e12
    clk = sampler.summary()
    out = {"tflops": round(tflops, 1), "sm_mhz": clk.get("sm_mhz"), "power_w_median": clk.get("power_w_median")}
    if clk.get("sm_mhz"):
        out["frac_of_nominal_at_that_clock"] = round(tflops / (sms * 128 * 2 * clk["sm_mhz"] * 1e6 / 1e12), 4)
    return out


# ------------------------------------------------------------ the metric's other rungs (N = 1 line)

def _sustained(fn, stream, dev, seconds: float, skip_s: float = 0.3, graph: bool = True) -> dict:
    """Run fn back to back for about `seconds`, CUDA events around the whole
    run on `stream`, NVML clocks and power sampled meanwhile. With `graph`,
    the launches are captured into a CUDA graph of about 2 ms of work and
    the graph is replayed, so host launch overhead (a Python call per
    launch) does not limit small problems; both arms of a comparison are
    timed the same way. A capture that fails falls back to direct launches."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(5):
        fn()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    per = max(e0.elapsed_time(e1) / 5e3, 1e-6)
    launch = fn
    per_call, how = 1, "direct launches"
    if graph:
        k = max(1, min(64, int(2e-3 / per)))
        try:
            g = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(stream)
            with torch.cuda.stream(side), torch.cuda.graph(g, stream=side):
                for _ in range(k):
                    fn()
            torch.cuda.synchronize(dev)
            g.replay()
            torch.cuda.synchronize(dev)
            launch, per_call, how = g.replay, k, f"CUDA graph of {k} launches, replayed"
        except Exception as exc:  # capture refused: time direct launches
            torch.cuda.synchronize(dev)
            how = f"direct launches (graph capture failed: {type(exc).__name__})"
    calls = max(2, int(seconds / (per * per_call)))
    sampler = ClockSampler(dev.index if dev.index is not None else 0, period_s=0.02)
    sampler.start()
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(calls):
            launch()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    sampler.stop()
    return {"reps": calls * per_call, "s": e0.elapsed_time(e1) / 1e3, "clocks": sampler.summary(),
            "power": sampler.power_stats(skip_s), "timing": how}


def _energy_mj(sampler: "ClockSampler"):
    """The device's NVML energy counter (mJ since the driver loaded), or None."""
    if not sampler.ok:
        return None
    try:
        return float(sampler.nv.nvmlDeviceGetTotalEnergyConsumption(sampler.h))
    except Exception:
        return None


def _energy(tflops: float, run: dict) -> dict:
    clk, pw = run["clocks"], run["power"]
    out = {"sm_mhz": clk.get("sm_mhz"), "reasons": clk.get("reasons"), "avg_w": pw.get("avg_w")}
    if clk.get("sm_mhz"):
        out["tflops_per_mhz"] = round(tflops / clk["sm_mhz"], 4)
    if pw.get("avg_w"):
        out["j_per_tflop"] = round(pw["avg_w"] / tflops, 4)
    return out


def _gemm_e2e(inputs, output, launch, flops: float, stream, steps: int = 3) -> dict:
    """The GEMM through the C ABI with host operands: every step copies the
    inputs from pinned host memory, runs the GEMM and copies D back, all on
    one stream between CUDA events."""
    import torch

    hin = [(t.cpu().pin_memory(), t) for t in inputs]
    hout = torch.empty(output.shape, dtype=output.dtype, pin_memory=True)

    def step():
        for h, d in hin:
            d.copy_(h, non_blocking=True)
        launch()
        hout.copy_(output, non_blocking=True)

    with torch.cuda.stream(stream):
        step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    s = e0.elapsed_time(e1) / 1e3
    return {"value": round(flops * steps / s / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": int(sum(t.numel() * t.element_size() for t in inputs)),
            "d2h_bytes_per_step": int(output.numel() * output.element_size()), "steps": steps,
            "note": "pinned host operands -> device, GEMM, D -> pinned host, on one stream, every step"}


def _rel_frob(a, b) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _gemm_case(kind: str, n: int, dev, stream, seed: int = 31) -> dict:
    """One square tensor-core GEMM of the ladder on configured operands:
    fp8 / nvfp4 from N(0,1) quantised as the rung configuration states
    (gplk.operands, TN, BF16 D); bf16 / f16 / tf32 from U[-1,1), i8 from
    uniform bytes (column-major NN, the reference's cublasGemmEx layout).
    Returns our launch through the C ABI, the same product through the
    library (cuBLAS / cuBLASLt via torch) with a view of its output in our
    D's storage order, the operands and D for the end-to-end copy, and
    labels."""
    import torch
    import torch.nn.functional as F
    import gplk
    from gplk import operands as O

    c = {"kind": kind, "n": n, "flops": 2.0 * n ** 3, "peak": NOMINAL_TFLOPS[kind]}
    if kind in ("fp8", "nvfp4"):
        xa = O.normal(n, n, seed, dev)
        if kind == "fp8":
            qa, sa = O.quantize_fp8(xa)
            del xa
            xb = O.normal(n, n, seed + 1, dev)
            qb, sb = O.quantize_fp8(xb)
            del xb
            scale_a, scale_b = torch.tensor([sa], device=dev), torch.tensor([sb], device=dev)
            D = torch.empty(n, n, dtype=torch.bfloat16, device=dev)  # column-major M x N as (N, M)
            fa, fb = qa.view(torch.float8_e4m3fn), qb.view(torch.float8_e4m3fn)
            c["ours"] = lambda: gplk.gemm_fp8_tn(qa, qb, D, scale_a, scale_b)
            c["library"] = lambda: torch._scaled_mm(fa, fb.t(), scale_a=scale_a, scale_b=scale_b,
                                                    out_dtype=torch.bfloat16)
            c["library_name"] = "cuBLASLt FP8 TN via torch._scaled_mm (per-tensor scales, BF16 out)"
            c["inputs"] = [qa, qb]
            c["dtype"] = "e4m3"
            c["workload"] = (f"FP8 E4M3 TN GEMM M=N=K={n}, N(0,1) operands, per-tensor amax/448 scales, "
                             "FP32 acc, BF16 out")
        else:
            qa, sfa, ga = O.quantize_nvfp4(xa)
            del xa
            xb = O.normal(n, n, seed + 1, dev)
            qb, sfb, gb = O.quantize_nvfp4(xb)
            del xb
            alpha = torch.tensor([ga * gb], device=dev)
            D = torch.empty(n, n, dtype=torch.bfloat16, device=dev)
            fa, fb = qa.view(torch.float4_e2m1fn_x2), qb.view(torch.float4_e2m1fn_x2)
            ssa = sfa.view(torch.float8_e4m3fn).view(n, n // 16)
            ssb = sfb.view(torch.float8_e4m3fn).view(n // 16, n)
            gat, gbt = torch.tensor([ga], device=dev), torch.tensor([gb], device=dev)
            rec = [F.ScalingType.BlockWise1x16, F.ScalingType.TensorWise]
            sw = [F.SwizzleType.SWIZZLE_32_4_4]
            c["ours"] = lambda: gplk.gemm_nvfp4_tn(qa, qb, sfa, sfb, D, n, alpha)
            c["library"] = lambda: F.scaled_mm(fa, fb.t(), [ssa, gat], rec, [ssb, gbt], rec, swizzle_a=sw,
                                               swizzle_b=sw, output_dtype=torch.bfloat16)
            c["library_name"] = "cuBLASLt NVFP4 (VEC16 UE4M3 block scales + per-tensor scales) via torch scaled_mm"
            c["inputs"] = [qa, qb, sfa, sfb]
            c["dtype"] = "e2m1"
            c["workload"] = (f"NVFP4 E2M1 TN GEMM M=N=K={n}, N(0,1) operands, UE4M3 per-16 block scales + "
                             "per-tensor FP32 scale, FP32 acc, BF16 out")
        c["lib_view"] = lambda out: out  # (M, N) row-major; ours is D.view(N, M).t()
        c["ours_view"] = lambda: D.view(n, n).t()
    else:
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        if kind == "i8":
            A = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
            B = torch.randint(-128, 128, (n, n), dtype=torch.int8, device=dev, generator=g)
            D = torch.empty(n, n, dtype=torch.int32, device=dev)
            c["library"] = lambda: torch._int_mm(B, A)
            c["library_name"] = "cuBLASLt INT8 via torch._int_mm (S32 out)"
        else:
            tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "tf32": torch.float32}[kind]
            A = (torch.rand(n, n, device=dev, generator=g) * 2 - 1).to(tdt)
            B = (torch.rand(n, n, device=dev, generator=g) * 2 - 1).to(tdt)
            D = torch.empty(n, n, dtype=tdt, device=dev)

            def library():
                if kind == "tf32":
                    torch.backends.cuda.matmul.allow_tf32 = True
                return torch.matmul(B, A)

            c["library"] = library
            c["library_name"] = f"cuBLAS {kind.upper()} via torch.matmul" + (" (TF32 allowed)" if kind == "tf32" else "")
        # Column-major A (M x K) is the row-major (K, M) tensor A; B likewise
        # (N, K); D stored (N, M) = B-rows x A-columns = torch.matmul(B, A).
        c["ours"] = lambda: gplk.gemm_nn(kind, A, B, D, n, n, n)
        c["lib_view"] = lambda out: out
        c["ours_view"] = lambda: D
        c["inputs"] = [A, B]
        c["dtype"], c["workload"] = NN_GEMMS[kind][0], NN_GEMMS[kind][1].replace("8192", str(n))
        if kind in ("bf16", "f16"):
            pk = measured_peaks()
            c["peak"] = pk["bf16_tflops"]
    c["D"] = D
    return c


def _case_extras(case: dict, stream, dev, seconds: float, ours_tflops: float, run: dict | None) -> dict:
    """The library's throughput on the same operands and GPU (sustained for
    `seconds`, with clocks and power), the relative Frobenius difference of
    the two outputs, and the GEMM end to end through the C ABI with host
    operands."""
    import torch

    lib = {"impl": case["library_name"]}
    try:
        ref = case["library"]()
        torch.cuda.synchronize(dev)
        case["ours"]()
        torch.cuda.synchronize(dev)
        lib["rel_frob_vs_ours"] = round(_rel_frob(case["ours_view"](), case["lib_view"](ref)), 6)
        del ref
        lrun = _sustained(case["library"], stream, dev, seconds)
        ltf = case["flops"] * lrun["reps"] / lrun["s"] / 1e12
        lib.update({"value": round(ltf, 1), "unit": "TFLOP/s", "timing": lrun["timing"], "clocks": lrun["clocks"],
                    "energy": _energy(ltf, lrun), "ours_over_library": round(ours_tflops / ltf, 4)})
    except Exception as exc:  # the library's kernel for this format may be missing from this torch build
        lib["unavailable"] = f"{type(exc).__name__}: {str(exc).splitlines()[0][:200]}"
    out = {"library": lib, "e2e": _gemm_e2e(case["inputs"], case["D"], case["ours"], case["flops"], stream)}
    if run is not None:
        out["energy"] = _energy(ours_tflops, run)
    return out


def _sustained_extras(case: dict, stream, dev, seconds: float) -> dict:
    """For a --workload GEMM line: ours sustained for `seconds` (the short
    timed region above runs before the power controller settles), then the
    library the same way, so `ours_over_library` compares like with like."""
    run = _sustained(case["ours"], stream, dev, seconds)
    tflops = case["flops"] * run["reps"] / run["s"] / 1e12
    out = {"sustained": {"value": round(tflops, 1), "unit": "TFLOP/s", "launches": run["reps"],
                         "seconds": round(run["s"], 3), "timing": run["timing"], "clocks": run["clocks"]}}
    out.update(_case_extras(case, stream, dev, seconds, tflops, run))
    return out


def rung_gemm(kind: str, dev, stream, seconds: float) -> dict:
    """FP8 E4M3 8192^3 or NVFP4 16384^3 on N(0,1) operands quantised as the
    rung configuration states, through the C ABI, sustained for `seconds`;
    the same operands through cuBLASLt on the same GPU beside it; and the
    GEMM end to end with host operands."""
    import gplk

    n = 8192 if kind == "fp8" else 16384
    case = _gemm_case(kind, n, dev, stream)
    run = _sustained(case["ours"], stream, dev, seconds)
    tflops = case["flops"] * run["reps"] / run["s"] / 1e12
    peak = case["peak"]
    out = {"metric": f"{kind} GEMM TFLOP/s", "value": round(tflops, 1), "unit": "TFLOP/s", "dtype": case["dtype"],
           "config": {"workload": case["workload"], "size": n, "l2": "operands larger than L2"},
           "launches": run["reps"], "seconds": round(run["s"], 3), "timing": run["timing"],
           "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(tflops / peak, 4), "peak_source": "nominal dense",
                        "traffic": NCU_TRAFFIC.get(kind)},
           "clocks": run["clocks"]}
    out.update(_case_extras(case, stream, dev, seconds, tflops, run))
    code, site = gplk.status_read()
    if code != 0:
        raise RuntimeError(f"device status {code} at {site:#x}")
    return out


def rung_power(dev, stream, seconds: float, mix=(4, 1, 2), budget_us: float = 1000.0) -> dict:
    """Sustained power of the powervirus kernel (time-boxed launches back to
    back) as a percentage of the enforced limit, beside the reference's
    strongest library rung on the same GPU: cuBLASLt FP8 8192^3 GEMMs back
    to back on operands filled with 0x38 (E4M3 1.0), as the reference's
    gpl_lt_init fills them."""
    import torch
    import gplk

    weights = list(mix) + [0] * (8 - len(mix))
    m, counts = gplk.pv_role_map(weights)
    role_map = torch.tensor(m, dtype=torch.uint8, device=dev)
    buf = torch.full((2 << 30,), 0x3C, dtype=torch.uint8, device=dev)
    sink = torch.zeros(1 + 1024, dtype=torch.float32, device=dev)
    cfg = gplk.PvCfg(role_map=role_map.data_ptr(), stream_buf=buf.data_ptr(), stream_bytes=buf.numel(),
                     sink=sink.data_ptr(), blocks=0, inner=256, budget_ns=int(budget_us * 1e3))
    idle = ClockSampler(dev.index if dev.index is not None else 0, period_s=0.02)
    torch.cuda.synchronize(dev)
    time.sleep(0.3)
    idle.start()
    time.sleep(0.5)
    idle.stop()
    idle_w = idle.power_stats().get("avg_w")
    run = _sustained(lambda: gplk.powervirus_launch(cfg, stream=stream), stream, dev, seconds, skip_s=0.5,
                     graph=False)  # 1 ms launches: no launch overhead to hide
    limit = run["power"].get("limit_w") or 1000.0
    lvl = run["power"].get("avg_w") or 0.0
    out = {"metric": "powervirus sustained power % of enforced limit", "value": round(100.0 * lvl / limit, 2),
           "unit": "%", "config": {"workload": "powervirus, continuous time-boxed launches: in-kernel tcgen05 FP8 + "
                                               "FFMA chains + TMA-bulk HBM streaming (2 GiB)",
                                   "mix_tensor_fma_dram": list(mix), "warps_per_64": counts,
                                   "launch_budget_us": budget_us},
           "launches": run["reps"], "seconds": round(run["s"], 3), "power": run["power"], "clocks": run["clocks"],
           "idle_w": idle_w, "swing_w": round(lvl - idle_w, 1) if idle_w else None, "enforced_limit_w": limit}
    del buf
    code, site = gplk.status_read()
    if code != 0:
        raise RuntimeError(f"device status {code} at {site:#x}")
    lib = {"impl": "cuBLASLt FP8 8192^3 TN GEMMs via torch._scaled_mm on 0x38 operands "
                   "(the reference's gpl_lt rung, tensor-only)"}
    try:
        n = 8192
        a = torch.full((n, n), 0x38, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn)
        b = torch.full((n, n), 0x38, dtype=torch.uint8, device=dev).view(torch.float8_e4m3fn)
        one = torch.ones(1, device=dev)
        lrun = _sustained(lambda: torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16),
                          stream, dev, seconds, skip_s=0.5, graph=False)
        llvl = lrun["power"].get("avg_w") or 0.0
        lib.update({"value": round(100.0 * llvl / limit, 2), "unit": "%", "power": lrun["power"],
                    "clocks": lrun["clocks"]})
        out["ours_minus_library_pct_points"] = round(out["value"] - lib["value"], 2)
    except Exception as exc:
        lib["unavailable"] = f"{type(exc).__name__}: {str(exc).splitlines()[0][:200]}"
    out["library"] = lib
    return out


def bench_rungs(args, dist: Dist) -> dict:
    """The metric's GEMM and power rungs, on this rank's GPU."""
    import torch

    dev = torch.device("cuda", dist.local)
    stream = torch.cuda.current_stream(dev)
    out = {}
    for kind in ("fp8", "nvfp4"):
        out[kind] = rung_gemm(kind, dev, stream, args.rung_seconds)
        torch.cuda.empty_cache()
    out["powervirus"] = rung_power(dev, stream, 2.0 * args.rung_seconds)
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------ fabric step beside the replicas (N > 1)

def fabric_check(dist: Dist, mib: int, steps: int, warmup: int) -> dict:
    """The powervirus cycle's fabric step on the replicas' GPUs: one
    gplk_fabric_allreduce_bf16 of `mib` MiB checked bit for bit against the
    same sum restated with torch (every rank's input gathered, added in FP32
    in rank order, rounded once to BF16), then timed beside NCCL's
    all_reduce on a buffer of the same size. Every rank takes the same
    collective steps; the verdict is agreed over all ranks."""
    import torch
    import gplk
    from gplk import rung
    from gplk.fabric import Fabric

    dev = torch.device("cuda", dist.local)
    count = (mib << 20) // 2
    fab = Fabric(dist.pg.group.WORLD, count * 2)
    buf = fab.tensor(count)
    g = torch.Generator(device=dev)
    g.manual_seed(11 + dist.rank)
    x = torch.randn(count, device=dev, generator=g).to(torch.bfloat16)
    parts = [torch.empty_like(x) for _ in range(dist.world)]
    dist.pg.all_gather(parts, x)
    want = parts[0].float()
    for p in parts[1:]:
        want = want + p.float()
    want = want.to(torch.bfloat16)
    del parts
    stream = torch.cuda.current_stream(dev)
    buf.copy_(x)
    torch.cuda.synchronize(dev)
    dist.barrier()
    fab.allreduce_bf16(count, stream=stream)
    torch.cuda.synchronize(dev)
    same = bool(torch.equal(buf.view(torch.int16), want.view(torch.int16)))
    bitexact = dist.sum(1.0 if same else 0.0) == dist.world
    del want
    other = x.clone()
    res = {}
    for name, fn in (("gplk", lambda: fab.allreduce_bf16(count, stream=stream)),
                     ("nccl", lambda: dist.pg.all_reduce(other))):
        buf.copy_(x)
        other.copy_(x)
        for _ in range(max(warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        dist.barrier()
        res[name] = dist.max(e0.elapsed_time(e1)) / steps
    # Watts: each implementation back to back for about 0.6 s (the same
    # count on every rank, from the max-over-ranks times above), this rank's
    # NVML power sampled and its energy counter read around the loop.
    nbytes = count * 2
    power = {}
    for name, fn in (("gplk", lambda: fab.allreduce_bf16(count, stream=stream)),
                     ("nccl", lambda: dist.pg.all_reduce(other))):
        iters = max(20, int(600.0 / res[name]))
        torch.cuda.synchronize(dev)
        dist.barrier()
        sampler = ClockSampler(dist.local, period_s=0.01)
        mj0 = _energy_mj(sampler)
        sampler.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        sampler.stop()
        mj1 = _energy_mj(sampler)
        dist.barrier()
        ms = dist.max(e0.elapsed_time(e1)) / iters
        avg_w = sampler.power_stats(skip_s=0.15).get("avg_w") or 0.0
        have = mj0 is not None and mj1 is not None
        mj_tot = dist.sum((mj1 - mj0) / iters if have else 0.0)
        all_have = dist.sum(1.0 if have else 0.0) == dist.world
        power[name] = {"steps": iters, "ms": round(ms, 4),
                       "busbw": round(rung.allreduce_busbw_gbs(nbytes, ms / 1e3, dist.world), 1),
                       "avg_w_per_gpu": round(dist.sum(avg_w) / dist.world, 1),
                       "mj_per_step_per_gpu": round(mj_tot / dist.world, 2) if all_have else None}
    code, site = gplk.status_read()
    dist.barrier()
    fab.close()
    status_ok = dist.sum(1.0 if code == 0 else 0.0) == dist.world
    bus = {k: rung.allreduce_busbw_gbs(nbytes, v / 1e3, dist.world) for k, v in res.items()}
    return {"impl": "gplk_fabric_allreduce_bf16 (NVLink peer loads/stores, no multicast)",
            "bytes": nbytes, "bitexact": bitexact, "status_ok": status_ok,
            "check": "every rank's seeded N(0,1) BF16 input gathered, summed in FP32 in rank order, rounded once",
            "ms_gplk": round(res["gplk"], 4), "busbw_gplk": round(bus["gplk"], 1),
            "ms_nccl": round(res["nccl"], 4), "busbw_nccl": round(bus["nccl"], 1),
            "gplk_over_nccl": round(res["nccl"] / res["gplk"], 4), "steps": steps,
            "sustained": power,
            "sustained_note": "about 0.6 s of back-to-back in-place allreduces per implementation; the buffer "
                              "saturates to +-inf after a few dozen in-place sums, the same for both; per-GPU "
                              "power and energy averaged over ranks"}


# ------------------------------------------------------------ powervirus rung

def node_power_summary(mon, on_ms: float, off_ms: float, phase: str) -> dict | None:
    """Node-level power from gplk_nodemon: the sum over all GPUs of the job,
    binned at 10 ms from the driver's buffered samples (device timestamps) and
    from the polled instantaneous path. The swing is p95 - p5 of the node sum."""
    if mon is None:
        return None
    if isinstance(mon, str):
        return {"unavailable": mon}
    from gplk import nodemon

    mon.stop()
    s = mon.samples()
    out = {"phase": phase, "devices": len(mon.devices), "period_ms": on_ms + off_ms}
    for name, src in (("buffered", nodemon.BUFFERED), ("polled", nodemon.POLLED)):
        n = int(((s["source"] == src)).sum())
        w = mon.node_series(src, t0=0.0, bin_s=0.01, max_bins=200000)
        w = w[10:] if len(w) > 20 else w  # drop the first 100 ms while every device starts reporting
        if n == 0 or len(w) == 0:
            out[name] = {"samples": n}
            continue
        pct = lambda q: float(sorted(w)[min(len(w) - 1, int(q * (len(w) - 1)))])  # noqa: E731
        out[name] = {"samples": n, "mean_w": round(float(w.mean()), 1), "p95_w": round(pct(0.95), 1),
                     "p5_w": round(pct(0.05), 1), "swing_w": round(pct(0.95) - pct(0.05), 1),
                     "max_w": round(float(w.max()), 1)}
    inst = s[(s["source"] == nodemon.POLLED) & (s["instant_w"] >= 0)]
    out["peak_instant_w_any_gpu"] = round(float(inst["instant_w"].max()), 1) if len(inst) else None
    mon.close()
    return out


def bench_powervirus(args, dist: Dist) -> dict:
    """Duty-cycled powervirus on every GPU in phase; each cycle = burst of
    time-boxed launches for duty_on_ms, a 256 MiB BF16 allreduce across all
    ranks (NCCL; skipped at N=1), then duty_off_ms idle. One step = one
    cycle. NVML power is sampled every 10 ms and split into burst and idle
    windows."""
    import torch
    import gplk
    from gplk import rung

    dev = torch.device("cuda", dist.local)
    torch.cuda.set_device(dev)
    gplk.lib()
    weights = [int(x) for x in args.mix.split(",")]
    weights += [0] * (8 - len(weights))
    m, counts = gplk.pv_role_map(weights)
    role_map = torch.tensor(m, dtype=torch.uint8, device=dev)
    buf = torch.full((2 << 30,), 0x3C, dtype=torch.uint8, device=dev)  # 2 GiB streaming buffer
    sink = torch.zeros(1 + 1024, dtype=torch.float32, device=dev)
    cfg = gplk.PvCfg()
    cfg.role_map = role_map.data_ptr()
    cfg.stream_buf = buf.data_ptr()
    cfg.stream_bytes = buf.numel()
    cfg.sink = sink.data_ptr()
    cfg.blocks = 0
    cfg.inner = 256
    cfg.budget_ns = int(args.budget_us * 1e3)
    stream = torch.cuda.current_stream(dev)
    ar_count = (args.fabric_mib << 20) // 2
    fab = None
    if dist.world > 1 and args.fabric == "gplk":
        from gplk.fabric import Fabric

        fab = Fabric(dist.pg.group.WORLD, ar_count * 2)
        ar = fab.tensor(ar_count)
        ar.fill_(1.0)
    else:
        ar = torch.ones((ar_count,), dtype=torch.bfloat16, device=dev)
    ar_bytes = ar.numel() * 2

    def launch():
        gplk.powervirus_launch(cfg, stream=stream)

    def sync():
        torch.cuda.synchronize(dev)

    staggered = args.phase == "staggered"
    if dist.world == 1 or staggered:
        step = None
    elif fab is not None:
        step = lambda: fab.allreduce_bf16(ar_count, stream=stream)  # noqa: E731
    else:
        step = lambda: dist.pg.all_reduce(ar)  # noqa: E731
    # The step is queued behind the burst's last launch (no host round trip)
    # and timed by CUDA events around it on the burst's stream.
    fab_ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))

    def allreduce_timed():
        fab_ev[0].record(stream)
        step()
        fab_ev[1].record(stream)

    allreduce = allreduce_timed if step is not None else None
    fabric_time = lambda: fab_ev[0].elapsed_time(fab_ev[1]) / 1e3  # noqa: E731
    on_ms, off_ms = args.duty_on_ms, args.duty_off_ms
    offset = rung.phase_offset_s(dist.rank, dist.world, on_ms, off_ms, staggered)
    rung.run_duty_cycles(max(args.warmup, 3), on_ms, off_ms, launch, sync, allreduce, barrier=dist.barrier,
                         fused=True, fabric_time=fabric_time)
    sampler = ClockSampler(dist.local, period_s=0.01)
    sampler.start()
    # Node-level view (rank 0): every GPU of the job sampled from one process
    # on one timebase, including the driver's buffered power samples.
    mon = None
    if dist.rank == 0:
        try:
            from gplk import nodemon

            mon = nodemon.NodeMonitor(list(range(dist.world)), hz=100, drain_ms=50)
        except Exception as exc:  # NVML or the sampler library unavailable: report without it
            mon = str(exc)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    e0.record(stream)
    log = rung.run_duty_cycles(args.steps, on_ms, off_ms, launch, sync, allreduce, barrier=dist.barrier,
                               start_offset_s=offset, fused=True, fabric_time=fabric_time)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    dist.barrier()
    sampler.stop()
    node = node_power_summary(mon, on_ms, off_ms, args.phase)
    code, site = gplk.status_read()
    if code != 0:
        raise RuntimeError(f"device status {code} at {site:#x}")
    ms_max = dist.max(e0.elapsed_time(e1))
    # NVML's power readings lag a 100 ms square wave by about one window, so
    # the level is read from the distribution of the samples: the burst
    # plateau is their 95th percentile, the idle floor their 5th.
    watts = sorted(w for (_t, _sm, _r, w) in sampler.samples)
    limit = sampler.limit_w or 1000.0

    def pct_at(q):
        return watts[min(len(watts) - 1, int(q * (len(watts) - 1)))] if watts else 0.0

    continuous = off_ms <= 0
    level_w = (sum(watts) / len(watts) if watts else 0.0) if continuous else pct_at(0.95)
    pct = 100.0 * level_w / limit
    pct_mean = dist.sum(pct) / dist.world
    node_level_w = dist.sum(level_w)
    fabric_s = sorted(log.fabric_s)[len(log.fabric_s) // 2] if log.fabric_s else 0.0
    clocks = sampler.summary()
    if fab is not None:
        torch.cuda.synchronize(dev)
        dist.barrier()
        fab.close()
    fabric_impl = "gplk_fabric_allreduce_bf16 (NVLink peer loads/stores)" if fab is not None else "NCCL all_reduce"
    fabric_launches = args.steps if fab is not None else 0
    return {
        "metric": "powervirus sustained power % of enforced limit" if continuous
        else "powervirus burst plateau (p95) power % of enforced limit",
        "value": round(pct_mean, 2), "unit": "%",
        "n_gpus": dist.world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3+f32", "data": "synthetic: 0x3c-filled 2 GiB stream, E4M3 1.0 tiles",
        "config": {"workload": "powervirus duty cycle: in-kernel tcgen05 FP8 + FFMA + TMA-bulk HBM streaming; "
                               f"{on_ms:g} ms on / {off_ms:g} ms off; {args.fabric_mib} MiB BF16 allreduce per cycle",
                   "mix_tensor_fma_dram_sfu_int32_smem_l2_atomic": weights, "warps_per_64": counts,
                   "launch_budget_us": args.budget_us,
                   "phase": args.phase,
                   "parallelism": f"replicas x{dist.world} in phase, {fabric_impl} per cycle"
                   if dist.world > 1 and not staggered else
                   (f"replicas x{dist.world} staggered over one period, no fabric step" if staggered
                    else "single GPU, no fabric step")},
        "power": {"level_w": round(level_w, 1), "avg_w": round(sum(watts) / len(watts), 1) if watts else None,
                  "p5_w": round(pct_at(0.05), 1), "p95_w": round(pct_at(0.95), 1),
                  "min_w": round(watts[0], 1) if watts else None, "max_w": round(watts[-1], 1) if watts else None,
                  "swing_p95_p5_w": round(pct_at(0.95) - pct_at(0.05), 1),
                  "node_level_sum_w": round(node_level_w, 1), "enforced_limit_w": limit,
                  "samples": len(watts), "source": "nvml instantaneous power, 10 ms"},
        "node": node,
        "fabric": {"impl": fabric_impl if allreduce else None,
                   "placement": "queued behind the burst's last launch (no host round trip); CUDA-event timed"
                   if allreduce else None,
                   "allreduce_bytes": ar_bytes if allreduce else 0, "median_s": round(fabric_s, 6),
                   "busbw_gbs": round(rung.allreduce_busbw_gbs(ar_bytes, fabric_s, dist.world), 1)
                   if allreduce else None},
        "clocks": clocks,
        "gpu_launches": int(sum(log.launches)) + fabric_launches,
    }


def pv_cycle(args, dist: Dist) -> dict:
    """A short in-phase powervirus duty cycle across all ranks (100 ms on /
    100 ms off, 6 timed cycles after 3 warm-up cycles, each ending in the
    gplk fabric step, 256 MiB BF16): per-rank power as % of the enforced
    limit (mean over ranks), node power from the driver's buffered samples,
    and the fabric step's time inside the cycle."""
    import copy

    a = copy.copy(args)
    a.steps, a.warmup = 6, 3
    a.duty_on_ms, a.duty_off_ms = 100.0, 100.0
    a.fabric, a.phase = "gplk", "aligned"
    full = bench_powervirus(a, dist)
    keep = ("metric", "value", "unit", "ms_per_step", "config", "power", "node", "fabric", "clocks", "gpu_launches")
    return {k: full[k] for k in keep if k in full}


# ------------------------------------------------------------ fabric step alone

def bench_fabric(args, dist: Dist) -> dict:
    """The powervirus cycle's fabric step on its own: an in-place BF16 sum
    allreduce of --fabric-mib MiB across all ranks, gplk_fabric_allreduce_bf16
    (value) against NCCL's all_reduce (reported beside it), CUDA events, max
    over ranks. Bus bandwidth follows NCCL's convention 2 (N-1)/N x bytes / t."""
    import torch

    if dist.world < 2:
        return {"metric": "fabric allreduce bus bandwidth", "unavailable": "needs 2 or more GPUs (torchrun)",
                "n_gpus": dist.world}
    torch.cuda.set_device(torch.device("cuda", dist.local))
    f = fabric_check(dist, args.fabric_mib, args.steps, args.warmup)
    if not f["status_ok"]:
        raise RuntimeError("fabric step recorded a device status")
    link = 770.0  # measured peer copy GB/s per direction per GPU on this pool
    return {
        "metric": "fabric allreduce bus bandwidth", "value": f["busbw_gplk"], "unit": "GB/s",
        "n_gpus": dist.world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": f["ms_gplk"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic N(0,1) BF16, seeded per rank",
        "config": {"workload": f"in-place BF16 sum allreduce of {args.fabric_mib} MiB per rank, one process per GPU",
                   "parallelism": f"allreduce x{dist.world}"},
        "nccl": {"ms_per_step": f["ms_nccl"], "busbw_gbs": f["busbw_nccl"]},
        "fabric": f,
        "roofline": {"bound": "nvlink", "achieved": f["busbw_gplk"], "peak": link, "unit": "GB/s",
                     "frac": round(f["busbw_gplk"] / link, 4), "traffic": None,
                     "peak_source": "measured peer copy per direction (pool figure)"},
        "gpu_launches": args.steps,
    }


# ------------------------------------------------------------ reference arm

def bench_reference(args, dist: Dist) -> dict | None:
    if dist.rank != 0:
        return None
    if args.workload == "sgemm":
        # The reference's SGEMM runs on the GPU (cublasGemmEx); its CPU
        # counterpart is the host triple loop the parity oracle restates.
        cpu = cpu_sgemm_tflops(args.sgemm_n, min(args.cpu_seconds, 10.0))
        return {
            "impl": "reference", "metric": "sgemm TFLOP/s", "value": cpu["value"], "unit": "TFLOP/s",
            "n_gpus": dist.world, "steps": 1, "warmup": 0, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic, seeded",
            "config": {"workload": f"FP32 SGEMM C = A*B row-major, M=N=K={args.sgemm_n}, U[-1,1)"},
            "cpu_baseline": cpu,
            "e2e": {"value": cpu["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    if args.workload != "memstream":
        return {"impl": "reference", "unavailable": f"no host implementation of the {args.workload} rung in the "
                                                    "reference (its GEMMs run in cuBLAS / cuBLASLt on the GPU)"}
    sys.path.insert(0, str(REPO / "oracle"))
    import numpy as np
    import oracle

    n = 1 << 28
    b = oracle.uniform_f32(n, seed=101)
    c = oracle.uniform_f32(n, seed=202)
    a = np.empty_like(b)
    th = host_threads()
    for _ in range(max(args.warmup, 1)):
        oracle.triad_into(a, b, c, TRIAD_S, th)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.triad_into(a, b, c, TRIAD_S, th)
    el = time.perf_counter() - t0
    value = 12 * n * args.steps / el / 1e9
    sample = f"each step: one host triad over 3 x 2^28 FP32 (3 GiB) of the 3 x 2^30 workload"
    return {
        "impl": "reference", "metric": "memstream triad GB/s", "value": round(value, 2), "unit": "GB/s",
        "n_gpus": dist.world, "steps": args.steps, "warmup": max(args.warmup, 1),
        "ms_per_step": round(el * 1e3 / args.steps, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic: b, c ~ U[0,1) seeded, s = 3.0",
        "config": {"workload": "memstream STREAM triad a = b + 3.0*c, FP32, 3 x 2^30 elements (4 GiB each)",
                   "sampled_elements_per_step": n,
                   "scope": f"one host: the node's whole CPU triad throughput on {th} cores, whatever the number "
                            "of GPUs (rank 0 runs it; the value is per byte, a 3 x 2^28 sample of the workload)"},
        "cpu_baseline": {"value": round(value, 2), "unit": "GB/s", "cores": th, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse_args()
    if args.impl == "reference":
        # Host-only arm: no process group; under torchrun only rank 0 works.
        class _Ranks:
            rank = int(os.environ.get("RANK", "0"))
            world = int(os.environ.get("WORLD_SIZE", "1"))

        line = bench_reference(args, _Ranks())
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    dist = Dist(args.gpus)
    try:
        if args.workload == "memstream":
            line = bench_memstream(args, dist)
        elif args.workload in ("sgemm", "fp8", "nvfp4") or args.workload in NN_GEMMS:
            line = bench_gemm(args, dist)
        elif args.workload == "fabric":
            line = bench_fabric(args, dist)
        else:
            line = bench_powervirus(args, dist)
        if args.workload == "memstream" and dist.world == 1 and not args.no_rungs:
            line["rungs"] = bench_rungs(args, dist)
        if args.workload == "memstream" and dist.world > 1 and not args.no_fabric_check:
            line["fabric"] = fabric_check(dist, args.fabric_mib, steps=10, warmup=3)
        if args.workload == "memstream" and dist.world > 1 and not args.no_pv_cycle:
            line["powervirus_cycle"] = pv_cycle(args, dist)
        if dist.rank == 0 and not args.no_cpu and args.workload == "memstream":
            line["cpu_baseline"] = cpu_triad_gbps(args.cpu_seconds)
        dist.barrier()  # the other ranks wait for rank 0's host baseline
        if dist.rank == 0 and dist.world == 1 and not args.no_cpu and args.workload == "sgemm":
            line["cpu_baseline"] = cpu_sgemm_tflops(args.sgemm_n, min(args.cpu_seconds, 10.0))
        if dist.rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
