/*
 * workload_memstream.cu - STREAM triad rung on libgplk (drop-in for the
 * runner's workload_memstream.cu; same entry point, phases and accounting).
 *
 * Arrays as in the reference (runner/src/workload_memstream.cu:60-84):
 * size x size FP32 elements each, A and B shared (memset 0x3c), one C per
 * stream (zeroed). Each iteration is one gplk_triad_f32 launch per stream,
 * C = A + scalar * B, on the 128-bit vectorised kernel (one vector per
 * thread, blocks in address order). The
 * scalar is the reference's 0.5 unless GPL_TRIAD_SCALAR is set (the
 * measured configuration uses 3.0); GPL_TRIAD_KERNEL=bulk selects the
 * TMA-bulk-staged variant.
 */
#include "workload.h"

#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "gpl_fault.h"
#include "gplk.h"
#include "util.h"

#define MS_CUDA(x)                                                                   \
    do {                                                                             \
        cudaError_t _e = (x);                                                        \
        if (_e != cudaSuccess) {                                                     \
            ctx->error = cudaGetErrorString(_e);                                     \
            gpl_errf("CUDA: %s (at %s:%d)", ctx->error, __FILE__, __LINE__);         \
            rc = -1;                                                                 \
            goto cleanup;                                                            \
        }                                                                            \
    } while (0)

#define MS_GPLK(x)                                                                   \
    do {                                                                             \
        int _s = (x);                                                                \
        if (_s != GPLK_STATUS_OK) {                                                  \
            ctx->error = gplk_status_string(_s);                                     \
            gpl_errf("gplk: %s (at %s:%d)", ctx->error, __FILE__, __LINE__);         \
            rc = -1;                                                                 \
            goto cleanup;                                                            \
        }                                                                            \
    } while (0)

int gpl_workload_memstream_run(gpl_workload_ctx_t *ctx) {
    const gpl_args_t *a = ctx->args;
    const int ns = a->streams;
    const size_t n = (size_t)a->size * (size_t)a->size;
    const size_t bytes = n * sizeof(float);
    const char *sv = getenv("GPL_TRIAD_SCALAR");
    const float scalar = sv ? (float)atof(sv) : 0.5f;
    const char *kv = getenv("GPL_TRIAD_KERNEL");
    const int bulk = kv && !strcmp(kv, "bulk");
    int rc = 0;
    float *dA = NULL, *dB = NULL;
    float **dC = (float **)calloc((size_t)ns, sizeof(float *));
    cudaStream_t *st = (cudaStream_t *)calloc((size_t)ns, sizeof(cudaStream_t));
    uint64_t warm_iters = 0, steady_iters = 0, t0, deadline;
    bool aborted = false;
    if (!dC || !st) {
        ctx->error = "oom (host arrays)";
        free(dC);
        free(st);
        return -1;
    }

    if (gpl_fault_is("alloc")) {
        ctx->error = GPL_FAULT_ALLOC_MSG;
        gpl_errf("memstream: %s", ctx->error);
        rc = -1;
        goto cleanup;
    }
    MS_CUDA(cudaMalloc((void **)&dA, bytes));
    MS_CUDA(cudaMalloc((void **)&dB, bytes));
    MS_CUDA(cudaMemset(dA, 0x3c, bytes));
    MS_CUDA(cudaMemset(dB, 0x3c, bytes));
    for (int i = 0; i < ns; i++) {
        MS_CUDA(cudaMalloc((void **)&dC[i], bytes));
        MS_CUDA(cudaMemset(dC[i], 0, bytes));
        MS_CUDA(cudaStreamCreateWithFlags(&st[i], cudaStreamNonBlocking));
    }

#define LAUNCH(i) MS_GPLK(bulk ? gplk_triad_f32_bulk(dC[i], dA, dB, scalar, n, st[i]) \
                               : gplk_triad_f32(dC[i], dA, dB, scalar, n, st[i]))
    if (gpl_fault_is("launch")) {
        ctx->error = GPL_FAULT_LAUNCH_MSG;
        gpl_errf("memstream: %s", ctx->error);
        rc = -1;
        goto cleanup;
    }
    for (int i = 0; i < ns; i++) LAUNCH(i);  /* prime */
    MS_CUDA(cudaDeviceSynchronize());

    gpl_telemetry_set_phase(ctx->tele, GPL_PHASE_WARMUP);
    t0 = gpl_mono_ns();
    deadline = t0 + (uint64_t)(a->warmup_sec * 1e9);
    while (gpl_mono_ns() < deadline) {
        for (int i = 0; i < ns; i++) {
            LAUNCH(i);
            warm_iters++;
        }
        if (warm_iters % (uint64_t)(ns * 8) == 0) MS_CUDA(cudaDeviceSynchronize());
    }
    MS_CUDA(cudaDeviceSynchronize());
    ctx->iterations_warmup = warm_iters;

    gpl_telemetry_set_phase(ctx->tele, GPL_PHASE_STEADY);
    t0 = gpl_mono_ns();
    deadline = t0 + (uint64_t)(a->steady_sec * 1e9);
    while (gpl_mono_ns() < deadline) {
        for (int i = 0; i < ns; i++) {
            LAUNCH(i);
            steady_iters++;
        }
        if (steady_iters % (uint64_t)(ns * 8) == 0) {
            MS_CUDA(cudaDeviceSynchronize());
            if (a->stop_on_throttle && gpl_telemetry_throttled_now(ctx->tele)) {
                aborted = true;
                break;
            }
        }
    }
    MS_CUDA(cudaDeviceSynchronize());
#undef LAUNCH
    ctx->iterations_steady = steady_iters;
    ctx->compute_seconds_steady = (double)(gpl_mono_ns() - t0) / 1e9;
    ctx->aborted_on_throttle = aborted;
    {
        int code = 0, site = 0;
        MS_GPLK(gplk_status_read(&code, &site, 1));
        if (code != GPLK_STATUS_OK) {
            ctx->error = gplk_status_string(code);
            gpl_errf("memstream: device status %s at site 0x%x", ctx->error, site);
            rc = -1;
        }
    }

cleanup:
    for (int i = 0; i < ns; i++) {
        if (st[i]) cudaStreamDestroy(st[i]);
        if (dC[i]) cudaFree(dC[i]);
    }
    if (dA) cudaFree(dA);
    if (dB) cudaFree(dB);
    free(dC);
    free(st);
    return rc;
}
