/*
 * workload_powervirus.cu - the mixed-unit maximum-power rung on B200
 * (drop-in for the runner's workload_powervirus.cu; same entry point,
 * flags, phases, duty cycle, ramp and fixed-work mode as
 * runner/src/workload_powervirus.cu:478-668).
 *
 * Kernel: gplk_powervirus_launch, one persistent 32-warp block per SM
 * (the reference launched 4 x SMs blocks of 8 warps). The tensor role is
 * in-kernel tcgen05 (one thread issues FP8 MMAs into TMEM), replacing the
 * warp-synchronous wmma role. With --tensor-backend cublas the tensor role
 * leaves the kernel, as in the reference, and GEMMs run on a concurrent
 * stream with the reference's semantics (runner/src/workload_powervirus.cu:
 * 281-397): fp8/fp4 through gpl_lt_* (libgplk tcgen05 GEMMs, D = A^T B,
 * now including a working NVFP4); bf16/fp16/tf32/int8 through libgplk's
 * tcgen05 NN GEMMs with beta = 1 (C = A * B + C, "beta=1 keeps C live");
 * fp32 through libgplk's SIMT SGEMM with beta = 1 (true FP32: the
 * reference's cublasGemmEx here ran with CUBLAS_TENSOR_OP_MATH, which lets
 * cuBLAS round FP32 operands down for the tensor cores); fp64 through
 * cublasGemmEx with beta = 1, the one precision left on the library
 * (tcgen05 has no FP64 kind). Ramped duty edges shape the kernel's block
 * count.
 */
#include "workload.h"

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "fabric_step.h"
#include "gemm_lt.h"
#include "gpl_fault.h"
#include "gplk.h"
#include "util.h"

namespace {

struct TensorStream {
    gpl_lt_gemm_t lt;
    bool use_lt = false;
    bool use_gplk = false;  // libgplk GEMM of the rung's precision (all but fp64)
    gpl_prec_t prec = GPL_PREC_FP16;
    cublasHandle_t h = nullptr;
    cudaStream_t stream = nullptr;
    void *dA = nullptr, *dB = nullptr, *dC = nullptr;
    void *dW = nullptr;  // fp32 SGEMM stream-K workspace
    size_t ws_bytes = 0;
    int n = 0;
    cudaDataType in_t = CUDA_R_16F, out_t = CUDA_R_16F;
    cublasComputeType_t comp_t = CUBLAS_COMPUTE_16F;
    bool active = false;
};

int tensor_stream_init(gpl_workload_ctx_t *ctx, TensorStream *ts) {
    const gpl_args_t *a = ctx->args;
    ts->n = a->size > 0 ? a->size : 4096;
    if (cudaStreamCreate(&ts->stream) != cudaSuccess) {
        ctx->error = "tensor stream create failed";
        return -1;
    }
    if (gpl_lt_precision_supported(a->precision)) {
        if (gpl_lt_init(&ts->lt, a->precision, ts->n, ts->stream) != 0) {
            ctx->error = "requested precision unavailable on this device";
            return -1;
        }
        ts->use_lt = true;
        ts->active = true;
        return 0;
    }
    size_t in_b = 2, out_b = 2;
    ts->prec = a->precision;
    ts->use_gplk = a->precision != GPL_PREC_FP64;
    switch (a->precision) {
        case GPL_PREC_FP32: ts->in_t = ts->out_t = CUDA_R_32F; ts->comp_t = CUBLAS_COMPUTE_32F; in_b = out_b = 4; break;
        case GPL_PREC_TF32: ts->in_t = ts->out_t = CUDA_R_32F; ts->comp_t = CUBLAS_COMPUTE_32F_FAST_TF32; in_b = out_b = 4; break;
        case GPL_PREC_BF16: ts->in_t = ts->out_t = CUDA_R_16BF; ts->comp_t = CUBLAS_COMPUTE_32F; break;
        case GPL_PREC_FP64: ts->in_t = ts->out_t = CUDA_R_64F; ts->comp_t = CUBLAS_COMPUTE_64F; in_b = out_b = 8; break;
        case GPL_PREC_INT8: ts->in_t = CUDA_R_8I; ts->out_t = CUDA_R_32I; ts->comp_t = CUBLAS_COMPUTE_32I; in_b = 1; out_b = 4; break;
        default: break;  // fp16
    }
    const size_t nn = (size_t)ts->n * ts->n;
    if (cudaMalloc(&ts->dA, nn * in_b) != cudaSuccess || cudaMalloc(&ts->dB, nn * in_b) != cudaSuccess ||
        cudaMalloc(&ts->dC, nn * out_b) != cudaSuccess) {
        ctx->error = "tensor stream: out of memory";
        return -1;
    }
    cudaMemset(ts->dA, 0x3c, nn * in_b);
    cudaMemset(ts->dB, 0x3c, nn * in_b);
    cudaMemset(ts->dC, 0, nn * out_b);
    if (ts->prec == GPL_PREC_FP32) {
        ts->ws_bytes = gplk_sgemm_workspace_bytes(ts->n, ts->n, ts->n);
        if (ts->ws_bytes && cudaMalloc(&ts->dW, ts->ws_bytes) != cudaSuccess) {
            ctx->error = "tensor stream: out of memory";
            return -1;
        }
    }
    if (ts->use_gplk) {
        ts->active = true;
        return 0;
    }
    if (cublasCreate(&ts->h) != CUBLAS_STATUS_SUCCESS) {
        ctx->error = "cublasCreate failed";
        return -1;
    }
    cublasSetStream(ts->h, ts->stream);
    cublasSetMathMode(ts->h, CUBLAS_TENSOR_OP_MATH);
    ts->active = true;
    return 0;
}

// `count` GEMMs on the tensor stream, asynchronous. beta = 1 keeps C live
// (C = A * B + C), as in the reference; the Lt formats write D = A^T B.
int tensor_stream_enqueue(TensorStream *ts, int count) {
    if (!ts->active || count <= 0) return 0;
    if (ts->use_lt) return gpl_lt_enqueue(&ts->lt, count);
    if (ts->use_gplk) {
        const int n = ts->n;
        for (int i = 0; i < count; i++) {
            int st = GPLK_STATUS_BAD_ARG;
            switch (ts->prec) {
                case GPL_PREC_BF16:
                    st = gplk_gemm_bf16_nn_acc((const uint16_t *)ts->dA, (const uint16_t *)ts->dB,
                                               (uint16_t *)ts->dC, n, n, n, ts->stream);
                    break;
                case GPL_PREC_FP16:
                    st = gplk_gemm_f16_nn_acc((const uint16_t *)ts->dA, (const uint16_t *)ts->dB,
                                              (uint16_t *)ts->dC, n, n, n, ts->stream);
                    break;
                case GPL_PREC_TF32:
                    st = gplk_gemm_tf32_nn_acc((const float *)ts->dA, (const float *)ts->dB, (float *)ts->dC, n, n,
                                               n, ts->stream);
                    break;
                case GPL_PREC_INT8:
                    st = gplk_gemm_i8_nn_acc((const int8_t *)ts->dA, (const int8_t *)ts->dB, (int32_t *)ts->dC, n,
                                             n, n, ts->stream);
                    break;
                default:  // fp32: column-major C = A * B + C is row-major C^T = B^T A^T + C^T
                    st = gplk_sgemm_f32((const float *)ts->dB, (const float *)ts->dA, (float *)ts->dC, n, n, n, n,
                                        n, n, 1.0f, ts->dW, ts->ws_bytes, ts->stream);
                    break;
            }
            if (st != GPLK_STATUS_OK) return -1;
        }
        return 0;
    }
    static const float f1 = 1.0f;
    static const double d1 = 1.0;
    static const int i1 = 1;
    static const unsigned short h1 = 0x3C00;
    const void *one = &f1;
    if (ts->comp_t == CUBLAS_COMPUTE_16F) one = &h1;
    else if (ts->comp_t == CUBLAS_COMPUTE_64F) one = &d1;
    else if (ts->comp_t == CUBLAS_COMPUTE_32I) one = &i1;
    for (int i = 0; i < count; i++) {
        if (cublasGemmEx(ts->h, CUBLAS_OP_N, CUBLAS_OP_N, ts->n, ts->n, ts->n, one, ts->dA, ts->in_t, ts->n, ts->dB,
                         ts->in_t, ts->n, one, ts->dC, ts->out_t, ts->n, ts->comp_t,
                         CUBLAS_GEMM_DEFAULT_TENSOR_OP) != CUBLAS_STATUS_SUCCESS)
            return -1;
    }
    return 0;
}

void tensor_stream_free(TensorStream *ts) {
    if (ts->use_lt) gpl_lt_free(&ts->lt);
    if (ts->h) cublasDestroy(ts->h);
    if (ts->stream) cudaStreamDestroy(ts->stream);
    if (ts->dA) cudaFree(ts->dA);
    if (ts->dB) cudaFree(ts->dB);
    if (ts->dC) cudaFree(ts->dC);
    if (ts->dW) cudaFree(ts->dW);
    ts->active = false;
}

void sleep_ms(double ms) {
    if (ms <= 0) return;
    struct timespec t;
    t.tv_sec = (time_t)(ms / 1000.0);
    t.tv_nsec = (long)((ms - (double)t.tv_sec * 1000.0) * 1e6);
    nanosleep(&t, NULL);
}

const char *role_label(int r) {
    static const char *names[GPLK_PV_ROLE_COUNT] = {"tensor", "fma", "dram", "sfu", "int32", "smem", "l2", "atomic"};
    return (r >= 0 && r < GPLK_PV_ROLE_COUNT) ? names[r] : "?";
}

}  // namespace

#define PV_CUDA(x)                                                                   \
    do {                                                                             \
        cudaError_t _e = (x);                                                        \
        if (_e != cudaSuccess) {                                                     \
            ctx->error = cudaGetErrorString(_e);                                     \
            gpl_errf("CUDA: %s (at %s:%d)", ctx->error, __FILE__, __LINE__);         \
            rc = -1;                                                                 \
            goto cleanup;                                                            \
        }                                                                            \
    } while (0)

#define PV_CHECK(cond, msg)                                                          \
    do {                                                                             \
        if (!(cond)) {                                                               \
            ctx->error = (msg);                                                      \
            gpl_errf("powervirus: %s (at %s:%d)", ctx->error, __FILE__, __LINE__);   \
            rc = -1;                                                                 \
            goto cleanup;                                                            \
        }                                                                            \
    } while (0)

int gpl_workload_powervirus_run(gpl_workload_ctx_t *ctx) {
    const gpl_args_t *a = ctx->args;
    const int ns = a->streams;
    const bool use_cublas_tensor = a->tensor_cublas && a->mix_tensor > 0;
    const int gemms_per_batch = use_cublas_tensor ? a->mix_tensor : 0;
    const bool run_kernel = !(use_cublas_tensor && a->mix_fma == 0 && a->mix_dram == 0);
    const int inner = a->size >= 4096 ? 2048 : 512;
    const int batch = 8;
    const bool duty = a->duty_on_ms > 0.0;
    const bool fixed_work = a->iters > 0;
    int rc = 0;
    int sm_count = 0;
    size_t freeb = 0, totalb = 0, buf_bytes = 0;
    float *d_stream = NULL, *d_sink = NULL;
    unsigned char *d_role = NULL;
    cudaStream_t *st = (cudaStream_t *)calloc((size_t)ns, sizeof(cudaStream_t));
    TensorStream ts;
    int w[GPLK_PV_ROLE_COUNT], counts[GPLK_PV_ROLE_COUNT];
    unsigned char role_map[GPLK_PV_ROLE_SLOTS];
    gplk_pv_cfg cfg;
    uint64_t t_start, s_start, warmup_ns, steady_ns, burst_ns;
    bool fabric = false;
    unsigned long long fabric_cycles = 0, cycles_done = 0;
    cudaEvent_t join[2] = {nullptr, nullptr};  // the other stream and the tensor stream, joined before the step
    memset(&cfg, 0, sizeof(cfg));
    PV_CHECK(st != NULL, "oom (streams)");

    PV_CHECK(!gpl_fault_is("alloc"), GPL_FAULT_ALLOC_MSG);
    PV_CUDA(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, a->device));
    PV_CUDA(cudaMemGetInfo(&freeb, &totalb));
    buf_bytes = freeb / 4;
    if (buf_bytes > ((size_t)2 << 30)) buf_bytes = (size_t)2 << 30;
    if (buf_bytes < ((size_t)64 << 20)) buf_bytes = (size_t)64 << 20;
    buf_bytes &= ~(size_t)0xFFF;
    PV_CUDA(cudaMalloc((void **)&d_stream, buf_bytes));
    PV_CUDA(cudaMalloc((void **)&d_role, GPLK_PV_ROLE_SLOTS));
    PV_CUDA(cudaMalloc((void **)&d_sink, sizeof(float) * (1 + 1024)));
    PV_CUDA(cudaMemset(d_stream, 0x3c, buf_bytes));
    PV_CUDA(cudaMemset(d_sink, 0, sizeof(float) * (1 + 1024)));

    if (use_cublas_tensor && tensor_stream_init(ctx, &ts) != 0) {
        rc = -1;
        goto cleanup;
    }
    {
        // The per-cycle fabric step (GPL_FABRIC=gplk|nccl): set up before the
        // phases start; the rendezvous aligns the ranks.
        const char *ferr = nullptr;
        PV_CHECK(gpl_fabric_step_init(&ferr) == 0, ferr);
        fabric = gpl_fabric_step_enabled() != 0;
        PV_CHECK(!fabric || duty, "fabric step: it runs once per duty cycle, so --duty-on-ms is required");
        PV_CHECK(!fabric || !fixed_work, "fabric step: --iters (fixed work) cannot keep the ranks in step");
        if (fabric) {
            fabric_cycles = gpl_fabric_cycles(a->steady_sec, a->duty_on_ms, a->duty_off_ms);
            for (int i = 0; i < (int)(sizeof join / sizeof join[0]); i++) PV_CUDA(cudaEventCreateWithFlags(
                &join[i], cudaEventDisableTiming));
            const gpl_fabric_stats_t *fs = gpl_fabric_stats();
            gpl_logf("  fabric step: %s BF16 allreduce of %.0f MiB, rank %d of %d, after each of %llu cycles%s",
                     fs->impl, fs->bytes / 1048576.0, fs->rank, fs->world, fabric_cycles,
                     a->stop_on_throttle ? " (--stop-on-throttle not honoured: the ranks stay in step)" : "");
        }
    }

    w[GPLK_PV_ROLE_TENSOR] = a->tensor_cublas ? 0 : a->mix_tensor;
    w[GPLK_PV_ROLE_FMA] = a->mix_fma;
    w[GPLK_PV_ROLE_DRAM] = a->mix_dram;
    w[GPLK_PV_ROLE_SFU] = a->mix_sfu;
    w[GPLK_PV_ROLE_INT32] = a->mix_int32;
    w[GPLK_PV_ROLE_SMEM] = a->mix_smem;
    w[GPLK_PV_ROLE_L2] = a->mix_l2;
    w[GPLK_PV_ROLE_ATOMIC] = a->mix_atomic;
    gplk_pv_build_role_map(w, role_map, counts);
    PV_CUDA(cudaMemcpy(d_role, role_map, GPLK_PV_ROLE_SLOTS, cudaMemcpyHostToDevice));
    {
        char mix[256];
        int off = 0;
        for (int r = 0; r < GPLK_PV_ROLE_COUNT; r++)
            if (counts[r] > 0 && off < (int)sizeof(mix) - 24)
                off += snprintf(mix + off, sizeof(mix) - off, "%s=%d ", role_label(r), counts[r]);
        gpl_logf("powervirus: %d blocks x %d warps | warps/%d: %s| stream=%.0f MiB", sm_count,
                 gplk_pv_block_threads() / 32, GPLK_PV_ROLE_SLOTS, mix, buf_bytes / 1048576.0);
        if (use_cublas_tensor)
            gpl_logf("  tensor backend: %s GEMM n=%d, %d per batch on a concurrent stream%s",
                     ts.use_lt ? "tcgen05 (libgplk gpl_lt)"
                     : !ts.use_gplk ? "cuBLAS fp64, beta = 1"
                     : ts.prec == GPL_PREC_FP32 ? "SIMT FP32 (libgplk), beta = 1"
                                                : "tcgen05 (libgplk), beta = 1",
                     ts.n, gemms_per_batch,
                     run_kernel ? "" : " (kernel disabled: tensor-only)");
        else
            gpl_logf("  tensor backend: in-kernel tcgen05 (single-thread issue)");
    }

    for (int i = 0; i < ns; i++) PV_CUDA(cudaStreamCreate(&st[i]));
    cfg.role_map = d_role;
    cfg.stream_buf = d_stream;
    cfg.stream_bytes = buf_bytes;
    cfg.sink = d_sink;
    cfg.blocks = sm_count;
    cfg.inner = inner;
    // Each role does exactly `inner` units per launch, as in the reference.
    // GPL_PV_BUDGET_US (fixed-time rungs only) instead time-boxes each launch:
    // every role keeps working until the budget has passed, so no unit idles
    // behind the slowest one. An always-ready FFMA warp can then crowd the
    // single MMA-issuing thread off its scheduler, so the budget suits
    // tensor-weighted mixes (e.g. tensor 2 : fma 1 : dram 1).
    {
        const char *bv = getenv("GPL_PV_BUDGET_US");
        const double us = bv ? atof(bv) : 0.0;
        cfg.budget_ns = (!fixed_work && us > 0.0) ? (unsigned long long)(us * 1e3) : 0ull;
    }

#define PV_KERNEL(nb, s)                                                                  \
    do {                                                                                  \
        cfg.blocks = (nb);                                                                \
        int _st = gplk_powervirus_launch(&cfg, (s));                                      \
        PV_CHECK(_st == GPLK_STATUS_OK, gplk_status_string(_st));                         \
    } while (0)
#define PV_TENSOR(count) PV_CHECK(tensor_stream_enqueue(&ts, (count)) == 0, "tensor stream enqueue failed")

    PV_CHECK(!gpl_fault_is("launch"), GPL_FAULT_LAUNCH_MSG);
    gpl_telemetry_set_phase(ctx->tele, GPL_PHASE_WARMUP);
    t_start = gpl_mono_ns();
    warmup_ns = (uint64_t)(a->warmup_sec * 1e9);
    while (gpl_mono_ns() - t_start < warmup_ns) {
        PV_TENSOR(gemms_per_batch * batch);
        if (run_kernel)
            for (int b = 0; b < batch; b++)
                for (int s = 0; s < ns; s++) PV_KERNEL(sm_count, st[s]);
        PV_CUDA(cudaDeviceSynchronize());
        ctx->iterations_warmup += (uint64_t)ns * batch;
    }

    gpl_telemetry_set_phase(ctx->tele, GPL_PHASE_STEADY);
    s_start = gpl_mono_ns();
    steady_ns = (uint64_t)(a->steady_sec * 1e9);
    burst_ns = (uint64_t)(a->duty_on_ms * 1e6);
    while (1) {
        if (fabric) {
            // A fixed number of cycles on every rank: each ends in a collective.
            if (cycles_done >= fabric_cycles) break;
        } else if (fixed_work) {
            if ((long long)ctx->iterations_steady >= a->iters) break;
        } else if (gpl_mono_ns() - s_start >= steady_ns) {
            break;
        }
        if (!fabric && a->stop_on_throttle && gpl_telemetry_throttled_now(ctx->tele)) {
            ctx->aborted_on_throttle = true;
            break;
        }
        if (duty) {
            // Burst for duty_on_ms, then a genuinely idle gap. A ramped edge
            // raises (and lowers) the block count over ramp_ns.
            const uint64_t b0 = gpl_mono_ns();
            uint64_t ramp_ns = 0;
            if (a->duty_ramp != GPL_RAMP_NONE) {
                ramp_ns = (uint64_t)((a->duty_ramp_ms > 0.0 ? a->duty_ramp_ms : a->duty_on_ms * 0.25) * 1e6);
                if (ramp_ns > burst_ns / 2) ramp_ns = burst_ns / 2;
            }
            uint64_t launch_ns = 0;  // fabric step: duration of the previous launch
            while (fabric || gpl_mono_ns() - b0 < burst_ns) {
                const uint64_t tl = gpl_mono_ns();
                int nb = sm_count;
                if (ramp_ns > 0) {
                    const uint64_t el = gpl_mono_ns() - b0;
                    double f = 1.0;
                    if (el < ramp_ns) {
                        const double x = (double)el / (double)ramp_ns;
                        f = a->duty_ramp == GPL_RAMP_EXP ? x * x : x;
                    } else if (el > burst_ns - ramp_ns) {
                        const double x = (double)(burst_ns - el) / (double)ramp_ns;
                        f = a->duty_ramp == GPL_RAMP_EXP ? x * x : x;
                    }
                    nb = (int)(sm_count * f);
                    if (nb < 1) nb = 1;
                }
                PV_TENSOR(gemms_per_batch);
                if (run_kernel)
                    for (int s = 0; s < ns; s++) PV_KERNEL(nb, st[s]);
                ctx->iterations_steady += (uint64_t)ns;
                // With a fabric step, the launch that reaches the end of the
                // burst is not waited for: the step is queued right behind
                // it, so the GPU goes from burst to allreduce with no host
                // round trip in between.
                if (fabric && tl - b0 + launch_ns >= burst_ns) break;
                PV_CUDA(cudaDeviceSynchronize());
                launch_ns = gpl_mono_ns() - tl;
            }
            if (fabric) {
                // The step goes on the first kernel stream (the tensor
                // stream when there is no kernel), after every other stream's
                // last work of the burst.
                cudaStream_t s0 = run_kernel ? st[0] : ts.stream;
                if (run_kernel)
                    for (int s = 1; s < ns; s++) {
                        PV_CUDA(cudaEventRecord(join[0], st[s]));
                        PV_CUDA(cudaStreamWaitEvent(s0, join[0], 0));
                    }
                if (run_kernel && ts.active) {
                    PV_CUDA(cudaEventRecord(join[1], ts.stream));
                    PV_CUDA(cudaStreamWaitEvent(s0, join[1], 0));
                }
                PV_CHECK(gpl_fabric_step_enqueue(s0) == 0, "fabric step: enqueue failed");
                PV_CUDA(cudaDeviceSynchronize());
                gpl_fabric_step_record();
                cycles_done++;
            }
            sleep_ms(a->duty_off_ms);
        } else {
            PV_TENSOR(gemms_per_batch * batch);
            if (run_kernel)
                for (int b = 0; b < batch; b++)
                    for (int s = 0; s < ns; s++) PV_KERNEL(sm_count, st[s]);
            PV_CUDA(cudaDeviceSynchronize());
            ctx->iterations_steady += (uint64_t)ns * batch;
        }
    }
    ctx->compute_seconds_steady = (double)(gpl_mono_ns() - s_start) / 1e9;
    {
        int code = 0, site = 0;
        PV_CHECK(gplk_status_read(&code, &site, 1) == GPLK_STATUS_OK, "gplk status read failed");
        if (code != GPLK_STATUS_OK) {
            ctx->error = gplk_status_string(code);
            gpl_errf("powervirus: device status %s at site 0x%x", ctx->error, site);
            rc = -1;
        }
    }
#undef PV_KERNEL
#undef PV_TENSOR

cleanup:
    gpl_fabric_step_free();
    for (int i = 0; i < (int)(sizeof join / sizeof join[0]); i++)
        if (join[i]) cudaEventDestroy(join[i]);
    tensor_stream_free(&ts);
    if (st) {
        for (int i = 0; i < ns; i++)
            if (st[i]) cudaStreamDestroy(st[i]);
        free(st);
    }
    if (d_stream) cudaFree(d_stream);
    if (d_role) cudaFree(d_role);
    if (d_sink) cudaFree(d_sink);
    return rc;
}
