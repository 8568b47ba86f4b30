/*
 * gemm_lt.h - drop-in replacement for the runner's cuBLASLt GEMM wrapper
 * (runner/src/gemm_lt.h:17-43 in the gpu-power-lab tree), implemented in
 * libgplk.so on the sm_100a tcgen05 GEMMs of include/gplk.h.
 *
 * Same four entry points, same return conventions (0 / -1, errors logged on
 * stderr), same public buffer fields with the same meaning, so callers that
 * seed operands through g->dA / g->dB / g->dScaleA / g->dScaleB and read
 * g->dD keep working:
 *   dA, dB     n x n operands, K-major (cuBLASLt TN: A is K x M column-major)
 *              E4M3 bytes for FP8; packed E2M1 (two per byte) for FP4
 *   dC, dD     n x n BF16, column-major (dC is allocated and zeroed as in the
 *              reference; D = result)
 *   dScaleA/B  per-tensor FP32 scales (FP8: D = sA * sB * A^T B)
 *   dScaleD    allocated for layout compatibility (unused, as in the reference)
 * Added for FP4, which the reference could not run (it set no block scales):
 *   dSFA/dSFB  UE4M3 block scales, one per 16 K-elements, in cuBLASLt's
 *              VEC16_UE4M3 layout (gplk_nvfp4_sf_bytes(n, n) bytes each)
 *   dAlpha     FP32 global scale product (D = alpha * sum sfa*a*sfb*b)
 * The cuBLASLt handle/descriptor members are gone; `ready`, `n`, `prec`,
 * `stream` keep their meaning. `workspace` / `workspace_bytes` hold K-padded
 * copies of the operands when n is not a multiple of 16 (FP8) or 256 (FP4);
 * each enqueue then refreshes them from dA / dB / dSFA / dSFB first.
 * The struct's layout differs from the reference's (whose cuBLASLt members
 * come first), so the drop-in is source-compatible: callers rebuild against
 * this header; code that touches only the named fields is unchanged.
 */
#ifndef GPL_GEMM_LT_H
#define GPL_GEMM_LT_H

#include <cuda_runtime_api.h>
#include <stdbool.h>
#include <stddef.h>

/* Inside the runner tree gpl_prec_t comes from its args.h; standalone, the
 * same enumerators are declared here (values of runner/src/args.h:31-40). */
#if defined(__has_include)
#if __has_include("args.h")
#include "args.h"
#endif
#endif
#ifndef GPL_ARGS_H
typedef enum {
    GPL_PREC_FP32 = 1,
    GPL_PREC_TF32,
    GPL_PREC_FP16,
    GPL_PREC_BF16,
    GPL_PREC_FP8,
    GPL_PREC_FP64,
    GPL_PREC_INT8,
    GPL_PREC_FP4,
} gpl_prec_t;
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    void *dA, *dB, *dC, *dD;
    void *dScaleA, *dScaleB, *dScaleD;
    void *dSFA, *dSFB, *dAlpha;
    void *workspace;
    size_t workspace_bytes;

    cudaStream_t stream;
    int n;
    gpl_prec_t prec;
    bool ready;
} gpl_lt_gemm_t;

/* True for FP8 (E4M3) and FP4 (NVFP4) on an sm_100 device.
 * Replaces runner/src/gemm_lt.cu:49-55. */
bool gpl_lt_precision_supported(gpl_prec_t p);

/* Allocates the n x n problem, fills A and B with 0x38 (E4M3 1.0; FP4 pair
 * -0 / 1.5), zeroes C, sets the scales (and FP4 block scales) to 1.0.
 * FP8 takes any n > 0, as the reference does; FP4 any multiple of 32.
 * Returns 0, or -1 with a logged reason (bad precision, an FP4 n that is not
 * a multiple of 32, out of memory, device not sm_100).
 * Replaces runner/src/gemm_lt.cu:57-161. */
int gpl_lt_init(gpl_lt_gemm_t *g, gpl_prec_t prec, int n, cudaStream_t stream);

/* Enqueues `count` GEMMs on g->stream (asynchronous).
 * Replaces runner/src/gemm_lt.cu:164-179. */
int gpl_lt_enqueue(gpl_lt_gemm_t *g, int count);

/* Frees everything gpl_lt_init allocated. Replaces runner/src/gemm_lt.cu:181-194. */
void gpl_lt_free(gpl_lt_gemm_t *g);

#ifdef __cplusplus
}
#endif

#endif /* GPL_GEMM_LT_H */
