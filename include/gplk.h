/*
 * gplk.h - C ABI of libgplk, the B200 (sm_100a) kernel library behind the
 * gpu-power-lab load generators.
 *
 * Every entry point:
 *   - takes plain device pointers, sizes and a CUDA stream;
 *   - is stream-ordered (asynchronous: a device fault or a device-side
 *     wait timeout shows up at the caller's next sync and in
 *     gplk_status_read) and allocates no device memory; the one exception
 *     is named where it occurs: gplk_fabric_create* allocate the fabric's
 *     buffers;
 *   - returns a gplk_status code synchronously from argument and launch
 *     checks.
 *
 * The reference path each launcher replaces is cited beside it
 * (paths relative to the gpu-power-lab source tree).
 */
#ifndef GPLK_H
#define GPLK_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    GPLK_STATUS_OK = 0,
    GPLK_STATUS_BAD_ARG = 1,        /* a size, alignment or pointer check failed */
    GPLK_STATUS_LAUNCH_FAIL = 2,    /* cudaLaunch / attribute call failed */
    GPLK_STATUS_DEVICE_TIMEOUT = 3, /* a bounded device-side wait ran out */
    GPLK_STATUS_UNSUPPORTED = 4,    /* device is not sm_100 or lacks a feature */
    GPLK_STATUS_CUDA_ERROR = 5      /* any other CUDA runtime error */
} gplk_status;

/* Human-readable name of a gplk_status value (static storage). */
const char *gplk_status_string(int status);

/* ABI version: bumped when a signature or a data layout changes. */
int gplk_abi_version(void);  /* 3: gplk_sgemm_f32 takes beta and a workspace */

/* Reads the device status word of the current device (first error recorded
 * by any gplk kernel since the last clear) and the site that recorded it.
 * Synchronises the current device. If clear != 0 the word is reset to OK. */
int gplk_status_read(int *code, int *site, int clear);

/* Watchdog self-test (no counterpart in the reference, which has no bounded
 * waits): one block waits on a barrier that nothing completes, gives up after
 * budget_ns (at most 2 s), writes 1 to *gave_up (device pointer, may be NULL)
 * and records GPLK_STATUS_DEVICE_TIMEOUT, site 0x0F01, in the status word.
 * The context stays usable. For tests of the failure path. */
int gplk_selftest_wait_timeout(unsigned long long budget_ns, int *gave_up, cudaStream_t stream);

/* ------------------------------------------------------------ memstream
 * STREAM triad a[i] = b[i] + s * c[i] in FP32, computed as one fused
 * multiply-add fmaf(s, c[i], b[i]) per element, so the result is bit-exact
 * against a host loop that calls fmaf.
 * Replaces stream_triad_kernel, runner/src/workload_memstream.cu:43-54
 * (launched at :102, :117, :140; its arrays are C = A + scalar * B).
 * a may not overlap b or c. n may be any size, including 0. */
int gplk_triad_f32(float *a, const float *b, const float *c, float s, size_t n,
                   cudaStream_t stream);

/* Same triad, with the operands staged through shared memory by 1-D TMA bulk
 * copies (cp.async.bulk) and the result written back by bulk stores.
 * Requires a, b, c 16-byte aligned. */
int gplk_triad_f32_bulk(float *a, const float *b, const float *c, float s, size_t n,
                        cudaStream_t stream);

/* dst[i] = src[i], FP32, 128-bit vectorised (the STREAM "copy" kernel). */
int gplk_copy_f32(float *dst, const float *src, size_t n, cudaStream_t stream);

/* ------------------------------------------------------------ SGEMM
 * C = A * B + beta * C in true FP32 (SIMT FFMA, no TF32), row-major:
 * A is M x K (leading dimension lda), B is K x N (ldb), C is M x N (ldc).
 * beta = 0 never reads C; otherwise each output is fmaf(beta, C_old, A*B),
 * which for beta = 1 is the sum rounded once.
 * Replaces cublasGemmEx with CUBLAS_COMPUTE_32F / CUBLAS_DEFAULT_MATH,
 * runner/src/workload_gemm.c:155-163, :174-179, :199-204 (column-major
 * C = A * B there, beta 0, which is the row-major product C^T = B^T * A^T
 * here), and the fp32 powervirus tensor stream's beta = 1 call,
 * runner/src/workload_powervirus.cu:363-380.
 * Problems whose 128 x 128 tiles leave a wave of SMs ragged run stream-K (a
 * cooperative launch, one block per SM) in the caller's workspace of
 * gplk_sgemm_workspace_bytes(M, N, K) bytes (16-byte aligned; 0 when the
 * shape does not use stream-K on the current device). With no workspace,
 * or a smaller one, the same product runs on whole tiles instead (the sums
 * then differ by FP32 rounding order). The first call that sees a workspace
 * zeroes its flags on `stream`; one workspace serves one stream at a time.
 * After a GPLK_STATUS_DEVICE_TIMEOUT at site 0x0B01 (a stream-K partial
 * that never arrived), zero the workspace before reusing it in a captured
 * CUDA graph, or re-instantiate the graph. */
size_t gplk_sgemm_workspace_bytes(int M, int N, int K);
int gplk_sgemm_f32(const float *A, const float *B, float *C, int M, int N, int K, int lda, int ldb, int ldc,
                   float beta, void *workspace, size_t workspace_bytes, cudaStream_t stream);

/* ------------------------------------------------------------ FP8 GEMM
 * D = (*scale_a) * (*scale_b) * (A^T * B) with E4M3 operands, FP32
 * accumulation and BF16 output, in cuBLASLt's TN convention:
 *   A: K x M column-major (each of the M rows holds K contiguous bytes),
 *   B: K x N column-major (each of the N columns holds K contiguous bytes),
 *   D: M x N column-major BF16 (ld = M).
 * scale_a / scale_b are device pointers to one FP32 each (per-tensor scales).
 * Replaces gpl_lt_enqueue's cublasLtMatmul for GPL_PREC_FP8,
 * runner/src/gemm_lt.cu:164-179 with the descriptor of :98-132.
 * Requires K % 16 == 0 and 16-byte aligned A and B; M and N are free. */
int gplk_gemm_fp8_tn(const uint8_t *A, const uint8_t *B, uint16_t *D, int M, int N, int K,
                     const float *scale_a, const float *scale_b, cudaStream_t stream);

/* ------------------------------------------------------------ NVFP4 GEMM
 * D = (*alpha) * sum_k (sfa[m, k/16] * a[m, k]) * (sfb[n, k/16] * b[n, k])
 * with E2M1 operands packed two per byte (element 2j in the low nibble of
 * byte j), one UE4M3 scale per 16 consecutive K-elements, FP32 accumulation
 * and BF16 output. A and B are K-major as for the FP8 GEMM (rows of K/2
 * bytes); D is M x N column-major BF16.
 * SFA / SFB use cuBLASLt's CUBLASLT_MATMUL_MATRIX_SCALE_VEC16_UE4M3 layout:
 * 128-row x 4-scale blocks of 512 bytes, block (r/128, kb/4) at byte offset
 * ((r/128) * ceil(K/64) + kb/4) * 512, and inside a block
 * (r % 32) * 16 + ((r % 128) / 32) * 4 + kb % 4. Row counts are padded to a
 * multiple of 128 and scale columns to a multiple of 4.
 * alpha is a device pointer to the FP32 product of the per-tensor scales.
 * This is the NVFP4 path that runner/src/gemm_lt.cu:76-82 tries to reach
 * (GPL_PREC_FP4) without block scales. Requires K % 256 == 0. */
int gplk_gemm_nvfp4_tn(const uint8_t *A, const uint8_t *B, const uint8_t *SFA,
                       const uint8_t *SFB, uint16_t *D, int M, int N, int K, const float *alpha,
                       cudaStream_t stream);

/* Bytes of one scale-factor array in the layout above, for `rows` rows and
 * a K extent of k elements. */
size_t gplk_nvfp4_sf_bytes(int rows, int k);

/* ------------------------------------------------------------ dense tensor-core GEMMs
 * C = A * B in the reference's cublasGemmEx layout: every matrix column-major,
 * no transposes, alpha = 1, beta = 0:
 *   A: M x K (ld = M), B: K x N (ld = K), D: M x N (ld = M).
 * Replaces cublasGemmEx(CUBLAS_OP_N, CUBLAS_OP_N, ...) at
 * runner/src/workload_gemm.c:155-163, :174-179, :199-204 for the precisions
 * that file maps at :44-79:
 *   bf16  BF16 in, FP32 accumulate, BF16 out   (CUDA_R_16BF, CUBLAS_COMPUTE_32F)
 *   f16   FP16 in, FP32 accumulate, FP16 out   (CUDA_R_16F, CUBLAS_COMPUTE_16F:
 *         the reference allows FP16 accumulation; this accumulates in FP32)
 *   tf32  FP32 in, TF32 products, FP32 out      (CUBLAS_COMPUTE_32F_FAST_TF32)
 *   i8    S8 in, S32 accumulate, S32 out        (CUDA_R_8I, CUBLAS_COMPUTE_32I)
 * Requires M and K multiples of 16 / element size (8 for bf16/f16, 4 for
 * tf32, 16 for i8) and 16-byte aligned A and B; N is free. */
int gplk_gemm_bf16_nn(const uint16_t *A, const uint16_t *B, uint16_t *D, int M, int N, int K,
                      cudaStream_t stream);
int gplk_gemm_f16_nn(const uint16_t *A, const uint16_t *B, uint16_t *D, int M, int N, int K,
                     cudaStream_t stream);
int gplk_gemm_tf32_nn(const float *A, const float *B, float *D, int M, int N, int K,
                      cudaStream_t stream);
int gplk_gemm_i8_nn(const int8_t *A, const int8_t *B, int32_t *D, int M, int N, int K,
                    cudaStream_t stream);

/* The same four with beta = 1: C = A * B + C in place (C is read, the
 * product added in FP32 / S32, the sum rounded once to C's type; S32 wraps).
 * Replaces the powervirus tensor stream's cublasGemmEx with beta = 1
 * ("beta=1 keeps C live"), runner/src/workload_powervirus.cu:363-380, for
 * bf16, fp16, tf32 and int8. Same layout and requirements as above. */
int gplk_gemm_bf16_nn_acc(const uint16_t *A, const uint16_t *B, uint16_t *C, int M, int N, int K,
                          cudaStream_t stream);
int gplk_gemm_f16_nn_acc(const uint16_t *A, const uint16_t *B, uint16_t *C, int M, int N, int K,
                         cudaStream_t stream);
int gplk_gemm_tf32_nn_acc(const float *A, const float *B, float *C, int M, int N, int K,
                          cudaStream_t stream);
int gplk_gemm_i8_nn_acc(const int8_t *A, const int8_t *B, int32_t *C, int M, int N, int K,
                        cudaStream_t stream);

/* ------------------------------------------------------------ fabric step
 * The powervirus cycle's fabric step: an in-place BF16 sum allreduce across
 * the GPUs of one node (one process per GPU), as one kernel over NVLink
 * peer memory. Replaces the ncclAllReduce of the multi-GPU rung
 * (runner/src/workload_nccl.cu:119-291), which the cycle issues on a 256 MiB
 * BF16 buffer. No multicast; plain peer loads and stores.
 *
 * Set-up, per rank, on its own device:
 *   1. gplk_fabric_create(rank, world, bytes, &f, handle): allocates this
 *      rank's buffer (bytes, a multiple of 16) and writes its CUDA IPC handle
 *      (gplk_fabric_handle_bytes() bytes) to `handle`;
 *   2. the caller exchanges the handles between ranks (all-gather, rank order);
 *   3. gplk_fabric_connect(f, handles): maps every peer's buffer.
 * gplk_fabric_data(f) is this rank's device buffer. Every rank then calls
 * gplk_fabric_allreduce_bf16(f, count, stream) in the same order: count BF16
 * elements (a multiple of 8) are summed in FP32 in rank order and rounded
 * once to BF16, in every rank's buffer. A rank that does not arrive within
 * 2 s makes the others return with GPLK_STATUS_DEVICE_TIMEOUT in the status
 * word (gplk_status_read). world <= 8. After such a timeout the ranks may
 * disagree on the fabric's epoch: destroy the fabric on every rank and
 * create a new one; do not reuse it. */
typedef struct gplk_fabric gplk_fabric;
size_t gplk_fabric_handle_bytes(void);
int gplk_fabric_create(int rank, int world, size_t bytes, gplk_fabric **out, void *handle);
int gplk_fabric_connect(gplk_fabric *f, const void *handles);
void *gplk_fabric_data(gplk_fabric *f);
int gplk_fabric_allreduce_bf16(gplk_fabric *f, size_t count, cudaStream_t stream);
/* The same with FP32 elements (count a multiple of 4), the reference NCCL
 * rung's data type (ncclFloat, runner/src/workload_nccl.cu:127-128). */
int gplk_fabric_allreduce_f32(gplk_fabric *f, size_t count, cudaStream_t stream);
/* Single process driving several GPUs, as the reference's NCCL rung does
 * (ncclCommInitAll over all devices, runner/src/workload_nccl.cu:18-23): one
 * fabric per listed device in out[0..ndev-1], buffers allocated on each
 * device and mapped through peer access (no IPC). Call the allreduce once
 * per fabric, each on a stream of that fabric's device; the call launches
 * on the fabric's device whatever device is current. */
int gplk_fabric_create_local(int ndev, const int *devices, size_t bytes, gplk_fabric **out);
int gplk_fabric_destroy(gplk_fabric *f);

/* ------------------------------------------------------------ powervirus */

#define GPLK_PV_ROLE_TENSOR 0  /* tcgen05 FP8 MMA into TMEM on smem-resident tiles */
#define GPLK_PV_ROLE_FMA 1     /* dependent FP32 FFMA chains */
#define GPLK_PV_ROLE_DRAM 2    /* HBM streaming by TMA bulk loads */
#define GPLK_PV_ROLE_SFU 3     /* transcendentals */
#define GPLK_PV_ROLE_INT32 4   /* integer multiply-add chains */
#define GPLK_PV_ROLE_SMEM 5    /* shared-memory read/write traffic */
#define GPLK_PV_ROLE_L2 6      /* L2-resident streaming */
#define GPLK_PV_ROLE_ATOMIC 7  /* atomics resolved in L2 */
#define GPLK_PV_ROLE_COUNT 8
#define GPLK_PV_ROLE_SLOTS 64  /* warp-slot map size */

typedef struct {
    const unsigned char *role_map; /* device, GPLK_PV_ROLE_SLOTS entries */
    const float *stream_buf;       /* device, HBM streaming source */
    size_t stream_bytes;           /* multiple of 16, >= 64 KiB */
    float *sink;                   /* device, 1 + 1024 floats (atomic targets) */
    float *verify_out;             /* device or NULL: one 32-bit word per thread (see below) */
    const uint8_t *mma_a;          /* device or NULL: 128 x 128 E4M3 tile, K-major */
    const uint8_t *mma_b;          /* device or NULL: 256 x 128 E4M3 tile, K-major */
    float *mma_out;                /* device or NULL: 128 x 256 F32 accumulator dump */
    int blocks;                    /* grid size; 0 = one block per SM */
    int inner;                     /* iterations of each role per launch */
    unsigned long long budget_ns;  /* 0: fixed work (exactly `inner` per role);
                                      else every role, after its fixed work,
                                      keeps going until budget_ns after its
                                      block started (uniform load) */
} gplk_pv_cfg;

/* One launch of the mixed-unit power kernel.
 * Replaces gpl_powervirus_kernel, runner/src/workload_powervirus.cu:100-249.
 * Blocks of gplk_pv_block_threads() threads (32 warps); warp w of block b
 * takes the role role_map[(2 * w + b % 2) % 64], so every block carries the
 * whole mix. With verify_out set, thread t of global warp g writes its role's
 * final 32-bit value (FMA chain sum bits, LCG xor, ...) to
 * verify_out[g * 32 + t] for bit-exact host checks; with mma_out set, block 0
 * dumps its 128 x 256 TMEM accumulator (row-major FP32) after `inner` tile
 * MMAs (each tile = A(128x128) x B(256x128)^T over K = 128). */
int gplk_powervirus_launch(const gplk_pv_cfg *cfg, cudaStream_t stream);

/* Largest-remainder apportionment of GPLK_PV_ROLE_SLOTS warp slots over the
 * eight role weights (runner/src/workload_powervirus.cu:414-454): a role
 * with a non-zero weight always gets at least one slot. Writes map[64] and
 * counts[8]. */
void gplk_pv_build_role_map(const int weights[GPLK_PV_ROLE_COUNT], unsigned char *map,
                            int *counts);

/* Threads per powervirus block (warps = value / 32). */
int gplk_pv_block_threads(void);

/* ------------------------------------------------------------ powervirus, no caller allocation
 * This entry point has no counterpart in the reference.
 *
 * The same kernel as gplk_powervirus_launch, for callers that cannot call
 * cudaMalloc: a load generator running inside another application's process
 * whose allocator owns the device memory, or a duty-cycled burst loop where
 * an allocation could synchronise the device mid-burst. The streaming
 * window (read by the DRAM and L2 roles) and the atomic sink live in one
 * static device array inside libgplk, held by every GPU that loads the
 * library until the process exits.
 *
 * The caller passes the inputs (role_map; optional mma_a/mma_b tiles) and the
 * outputs (optional verify_out, mma_out), as for gplk_powervirus_launch.
 * stream_bytes picks the window size: a multiple of 16 in
 * [64 KiB, GPLK_PV_NOALLOC_MAX_STREAM_BYTES]; a larger size is rejected with
 * GPLK_STATUS_BAD_ARG and a message on stderr. A 32 MiB window fits in L2,
 * so in this variant the DRAM role streams mostly from L2, not HBM.
 *
 * Every call, with the device current, resolves the array's device address
 * on that device and, ordered on `stream` before the launch, fills the window
 * with the byte 0x3c and zeroes the sink. Nothing is cached between calls
 * (the entry point stays valid after a cudaDeviceReset) and no call
 * synchronises. All calls share the array, so calls that overlap on the GPU
 * race on it. Allocates nothing: no cudaMalloc, cudaFree or allocating
 * library call. */
#define GPLK_PV_NOALLOC_MAX_STREAM_BYTES ((size_t)32 << 20)
int gplk_powervirus_launch_noalloc(const unsigned char *role_map, size_t stream_bytes, int blocks,
                                   int inner, float *verify_out, const uint8_t *mma_a,
                                   const uint8_t *mma_b, float *mma_out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GPLK_H */
