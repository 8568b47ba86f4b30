/*
 * workload_gemm.c - the GEMM ladder rung on B200 (drop-in for the runner's
 * workload_gemm.c; same entry point, loop structure and accounting).
 *
 *   fp32         gplk_sgemm_f32: true FP32 on the SIMT FFMA pipe, replacing
 *                cublasGemmEx(COMPUTE_32F, DEFAULT_MATH) at
 *                runner/src/workload_gemm.c:155-163
 *   fp8, fp4     gpl_lt_* from libgplk (tcgen05 E4M3 / NVFP4 GEMMs), which
 *                the reference rejected on this op (:84-89)
 *   bf16, fp16, tf32, int8
 *                gplk_gemm_{bf16,f16,tf32,i8}_nn: tcgen05 GEMMs on CTA pairs in
 *                the same column-major NN layout and output types as the
 *                reference's cublasGemmEx call (:45-79, :155-163)
 *   fp64         cublasGemmEx with the reference's type mapping: a plain
 *                library GEMM, the one precision left on it (tcgen05 has no
 *                FP64 kind)
 * The fp32 SGEMM's stream-K workspace (gplk_sgemm_workspace_bytes) is
 * allocated once per stream at set-up, beside the operands; the GEMM calls
 * in the timed loops allocate nothing.
 *
 * Square N x N x N problems, one C per stream, warm-up and steady phases by
 * wall clock, a device sync every 8 x streams launches (:167-219).
 */
#include "workload.h"

#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "gemm_lt.h"
#include "gpl_fault.h"
#include "gplk.h"
#include "util.h"

typedef struct {
    cublasHandle_t h;
    cudaDataType in_t, out_t;
    cublasComputeType_t comp_t;
    const void *alpha, *beta;
} gemm_cublas_t;

typedef enum { PATH_GPLK_SGEMM, PATH_GPLK_LT, PATH_GPLK_TC, PATH_CUBLAS } gemm_path_t;

static gemm_path_t path_for(gpl_prec_t p) {
    if (p == GPL_PREC_FP32) return PATH_GPLK_SGEMM;
    if (p == GPL_PREC_FP8 || p == GPL_PREC_FP4) return PATH_GPLK_LT;
    if (p == GPL_PREC_FP64) return PATH_CUBLAS;
    return PATH_GPLK_TC;
}

#define TC_SIZE_MSG \
    "size unsupported by the tcgen05 GEMM (a multiple of 8 for bf16/fp16, 4 for tf32, 16 for int8 is required)"

/* One tcgen05 GEMM of the rung's precision: column-major C = A * B. */
static int gplk_tc_gemm(gpl_prec_t p, const void *A, const void *B, void *C, int n, cudaStream_t s) {
    switch (p) {
        case GPL_PREC_BF16:
            return gplk_gemm_bf16_nn((const uint16_t *)A, (const uint16_t *)B, (uint16_t *)C, n, n, n, s);
        case GPL_PREC_FP16:
            return gplk_gemm_f16_nn((const uint16_t *)A, (const uint16_t *)B, (uint16_t *)C, n, n, n, s);
        case GPL_PREC_TF32:
            return gplk_gemm_tf32_nn((const float *)A, (const float *)B, (float *)C, n, n, n, s);
        case GPL_PREC_INT8:
            return gplk_gemm_i8_nn((const int8_t *)A, (const int8_t *)B, (int32_t *)C, n, n, n, s);
        default:
            return GPLK_STATUS_BAD_ARG;
    }
}

/* cublasGemmEx types for the precisions that stay on the library. */
static void cublas_types(gpl_prec_t p, gemm_cublas_t *g, size_t *in_bytes, size_t *out_bytes) {
    static const float f1 = 1.0f, f0 = 0.0f;
    static const double d1 = 1.0, d0 = 0.0;
    static const int i1 = 1, i0 = 0;
    static const unsigned short h1 = 0x3C00, h0 = 0x0000; /* binary16 1.0 and 0.0 */
    g->alpha = &f1;
    g->beta = &f0;
    switch (p) {
        case GPL_PREC_TF32:
            g->in_t = CUDA_R_32F; g->out_t = CUDA_R_32F; g->comp_t = CUBLAS_COMPUTE_32F_FAST_TF32;
            *in_bytes = 4; *out_bytes = 4;
            break;
        case GPL_PREC_FP16:
            g->in_t = CUDA_R_16F; g->out_t = CUDA_R_16F; g->comp_t = CUBLAS_COMPUTE_16F;
            g->alpha = &h1; g->beta = &h0;
            *in_bytes = 2; *out_bytes = 2;
            break;
        case GPL_PREC_BF16:
            g->in_t = CUDA_R_16BF; g->out_t = CUDA_R_16BF; g->comp_t = CUBLAS_COMPUTE_32F;
            *in_bytes = 2; *out_bytes = 2;
            break;
        case GPL_PREC_FP64:
            g->in_t = CUDA_R_64F; g->out_t = CUDA_R_64F; g->comp_t = CUBLAS_COMPUTE_64F;
            g->alpha = &d1; g->beta = &d0;
            *in_bytes = 8; *out_bytes = 8;
            break;
        case GPL_PREC_INT8:
        default:
            g->in_t = CUDA_R_8I; g->out_t = CUDA_R_32I; g->comp_t = CUBLAS_COMPUTE_32I;
            g->alpha = &i1; g->beta = &i0;
            *in_bytes = 1; *out_bytes = 4; /* 8-bit inputs into a 32-bit accumulator */
            break;
    }
}

int gpl_workload_gemm_run(gpl_workload_ctx_t *ctx) {
    const gpl_args_t *a = ctx->args;
    const int N = a->size, ns = a->streams;
    const gemm_path_t path = path_for(a->precision);
    const size_t nn = (size_t)N * (size_t)N;
    int rc = 0;
    uint64_t warm = 0, steady = 0, t0, deadline;
    bool aborted = false;
    void *dA = NULL, *dB = NULL;
    void **dC = (void **)calloc((size_t)ns, sizeof(void *));
    void **dW = (void **)calloc((size_t)ns, sizeof(void *)); /* SGEMM stream-K workspace per stream */
    size_t ws_bytes = 0;
    cudaStream_t *st = (cudaStream_t *)calloc((size_t)ns, sizeof(cudaStream_t));
    gemm_cublas_t *cb = (gemm_cublas_t *)calloc((size_t)ns, sizeof(gemm_cublas_t));
    gpl_lt_gemm_t *lt = (gpl_lt_gemm_t *)calloc((size_t)ns, sizeof(gpl_lt_gemm_t));
    if (!dC || !dW || !st || !cb || !lt) {
        ctx->error = "oom (host arrays)";
        rc = -1;
        goto cleanup;
    }

#define G_CUDA(x)                                                                   \
    do {                                                                            \
        cudaError_t _e = (x);                                                       \
        if (_e != cudaSuccess) {                                                    \
            ctx->error = cudaGetErrorString(_e);                                    \
            gpl_errf("CUDA: %s (at %s:%d)", ctx->error, __FILE__, __LINE__);        \
            rc = -1;                                                                \
            goto cleanup;                                                           \
        }                                                                           \
    } while (0)

    if (gpl_fault_is("alloc")) {
        ctx->error = GPL_FAULT_ALLOC_MSG;
        gpl_errf("gemm: %s", ctx->error);
        rc = -1;
        goto cleanup;
    }
    for (int i = 0; i < ns; i++) G_CUDA(cudaStreamCreateWithFlags(&st[i], cudaStreamNonBlocking));

    if (path == PATH_GPLK_LT) {
        for (int i = 0; i < ns; i++) {
            if (gpl_lt_init(&lt[i], a->precision, N, st[i]) != 0) {
                ctx->error = "requested precision unavailable on this device";
                rc = -1;
                goto cleanup;
            }
        }
    } else {
        size_t in_b = 4, out_b = 4;
        if (path != PATH_GPLK_SGEMM) cublas_types(a->precision, &cb[0], &in_b, &out_b);
        G_CUDA(cudaMalloc(&dA, nn * in_b));
        G_CUDA(cudaMalloc(&dB, nn * in_b));
        G_CUDA(cudaMemset(dA, 0x3c, nn * in_b));
        G_CUDA(cudaMemset(dB, 0x3c, nn * in_b));
        if (path == PATH_GPLK_SGEMM) ws_bytes = gplk_sgemm_workspace_bytes(N, N, N);
        for (int i = 0; i < ns; i++) {
            G_CUDA(cudaMalloc(&dC[i], nn * out_b));
            G_CUDA(cudaMemset(dC[i], 0, nn * out_b));
            if (ws_bytes) G_CUDA(cudaMalloc(&dW[i], ws_bytes));
            if (path == PATH_CUBLAS) {
                cb[i] = cb[0];
                if (cublasCreate(&cb[i].h) != CUBLAS_STATUS_SUCCESS ||
                    cublasSetStream(cb[i].h, st[i]) != CUBLAS_STATUS_SUCCESS) {
                    ctx->error = "cublas failure";
                    rc = -1;
                    goto cleanup;
                }
                cublasSetMathMode(cb[i].h, a->precision == GPL_PREC_TF32 ? CUBLAS_TF32_TENSOR_OP_MATH
                                                                         : CUBLAS_DEFAULT_MATH);
            }
        }
    }

    /* One GEMM on stream i. Column-major C = A * B (the reference's
     * convention) is the row-major product C^T = B^T * A^T for the SIMT
     * kernel; for these square fills the operand order is immaterial. */
#define ONE_GEMM(i)                                                                                     \
    do {                                                                                                \
        int _r = 0;                                                                                     \
        if (path == PATH_GPLK_SGEMM) {                                                                  \
            _r = gplk_sgemm_f32((const float *)dB, (const float *)dA, (float *)dC[i], N, N, N, N, N, N, \
                                0.0f, dW[i], ws_bytes, st[i]);                                          \
            if (_r) ctx->error = gplk_status_string(_r);                                                \
        } else if (path == PATH_GPLK_LT) {                                                              \
            _r = gpl_lt_enqueue(&lt[i], 1);                                                             \
            if (_r) ctx->error = "gemm_lt enqueue failed";                                              \
        } else if (path == PATH_GPLK_TC) {                                                              \
            _r = gplk_tc_gemm(a->precision, dA, dB, dC[i], N, st[i]);                                   \
            if (_r) ctx->error = _r == GPLK_STATUS_BAD_ARG ? TC_SIZE_MSG : gplk_status_string(_r);      \
        } else {                                                                                        \
            _r = cublasGemmEx(cb[i].h, CUBLAS_OP_N, CUBLAS_OP_N, N, N, N, cb[i].alpha, dA, cb[i].in_t,  \
                              N, dB, cb[i].in_t, N, cb[i].beta, dC[i], cb[i].out_t, N, cb[i].comp_t,   \
                              CUBLAS_GEMM_DEFAULT_TENSOR_OP) != CUBLAS_STATUS_SUCCESS;                   \
            if (_r) ctx->error = "cublas failure";                                                      \
        }                                                                                               \
        if (_r) {                                                                                       \
            gpl_errf("gemm: %s (at %s:%d)", ctx->error, __FILE__, __LINE__);                           \
            rc = -1;                                                                                    \
            goto cleanup;                                                                               \
        }                                                                                               \
    } while (0)

    if (gpl_fault_is("launch")) {
        ctx->error = GPL_FAULT_LAUNCH_MSG;
        gpl_errf("gemm: %s", ctx->error);
        rc = -1;
        goto cleanup;
    }
    for (int i = 0; i < ns; i++) ONE_GEMM(i); /* prime */
    G_CUDA(cudaDeviceSynchronize());

    gpl_telemetry_set_phase(ctx->tele, GPL_PHASE_WARMUP);
    t0 = gpl_mono_ns();
    deadline = t0 + (uint64_t)(a->warmup_sec * 1e9);
    while (gpl_mono_ns() < deadline) {
        for (int i = 0; i < ns; i++) {
            ONE_GEMM(i);
            warm++;
        }
        if (warm % (uint64_t)(ns * 8) == 0) G_CUDA(cudaDeviceSynchronize());
    }
    G_CUDA(cudaDeviceSynchronize());
    ctx->iterations_warmup = warm;

    gpl_telemetry_set_phase(ctx->tele, GPL_PHASE_STEADY);
    t0 = gpl_mono_ns();
    deadline = t0 + (uint64_t)(a->steady_sec * 1e9);
    while (gpl_mono_ns() < deadline) {
        for (int i = 0; i < ns; i++) {
            ONE_GEMM(i);
            steady++;
        }
        if (steady % (uint64_t)(ns * 8) == 0) {
            G_CUDA(cudaDeviceSynchronize());
            if (a->stop_on_throttle && gpl_telemetry_throttled_now(ctx->tele)) {
                aborted = true;
                break;
            }
        }
    }
    G_CUDA(cudaDeviceSynchronize());
    ctx->iterations_steady = steady;
    ctx->compute_seconds_steady = (double)(gpl_mono_ns() - t0) / 1e9;
    ctx->aborted_on_throttle = aborted;
    if (path != PATH_CUBLAS) {
        int code = 0, site = 0;
        if (gplk_status_read(&code, &site, 1) != GPLK_STATUS_OK || code != GPLK_STATUS_OK) {
            ctx->error = code ? gplk_status_string(code) : "gplk status read failed";
            gpl_errf("gemm: device status %s at site 0x%x", ctx->error, site);
            rc = -1;
        }
    }
#undef ONE_GEMM
#undef G_CUDA

cleanup:
    for (int i = 0; i < ns; i++) {
        if (lt && lt[i].ready) gpl_lt_free(&lt[i]);
        if (cb && cb[i].h) cublasDestroy(cb[i].h);
        if (st && st[i]) cudaStreamDestroy(st[i]);
        if (dC && dC[i]) cudaFree(dC[i]);
        if (dW && dW[i]) cudaFree(dW[i]);
    }
    if (dA) cudaFree(dA);
    if (dB) cudaFree(dB);
    free(dC);
    free(dW);
    free(st);
    free(cb);
    free(lt);
    return rc;
}
