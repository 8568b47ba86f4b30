// ref_shim.cu - exposes pieces of the reference runner, compiled from the
// reference's own sources (ref_build.sh), to the parity tests. TEST
// INFRASTRUCTURE ONLY: this is the checker, never the product.
//
// The reference keeps its triad kernel and role-map builder `static` inside
// runner/src/workload_memstream.cu and runner/src/workload_powervirus.cu, so
// this file includes those sources textually and adds extern "C" entry
// points around them. The runner's NVML sampler is not built; its two
// functions the workloads call are stubbed below.
#include "workload_memstream.cu"
#include "workload_powervirus.cu"

extern "C" {

void gpl_telemetry_set_phase(gpl_telemetry_t *t, gpl_phase_t p) { (void)t; (void)p; }
bool gpl_telemetry_throttled_now(gpl_telemetry_t *t) { (void)t; return false; }

// stream_triad_kernel (workload_memstream.cu:43-54) with the reference's
// launch geometry (:94-97): ceil(n/256) blocks of 256 threads, C = A + s*B.
int ref_triad_launch(float *C, const float *A, const float *B, float scalar, size_t n,
                     cudaStream_t stream) {
    const int threads = 256;
    const unsigned int blocks = (unsigned int)((n + threads - 1) / threads);
    if (n == 0) return 0;
    stream_triad_kernel<<<blocks, threads, 0, stream>>>(C, A, B, scalar, n);
    return (int)cudaGetLastError();
}

// build_role_map (workload_powervirus.cu:414-454) on a gpl_args_t holding
// the eight mix weights in role order.
void ref_build_role_map(const int w[8], int tensor_cublas, unsigned char *map, int *counts) {
    gpl_args_t a;
    gpl_args_defaults(&a);
    a.tensor_cublas = tensor_cublas != 0;
    a.mix_tensor = w[0];
    a.mix_fma = w[1];
    a.mix_dram = w[2];
    a.mix_sfu = w[3];
    a.mix_int32 = w[4];
    a.mix_smem = w[5];
    a.mix_l2 = w[6];
    a.mix_atomic = w[7];
    build_role_map(&a, map, counts);
}

// gpl_workload_{flops,bytes}_per_iter (workload_util.c:20-58).
double ref_flops_per_iter(int op, int prec, int size) {
    gpl_args_t a;
    gpl_args_defaults(&a);
    a.op = (gpl_op_t)op;
    a.precision = (gpl_prec_t)prec;
    a.size = size;
    return gpl_workload_flops_per_iter(&a);
}

double ref_bytes_per_iter(int op, int size) {
    gpl_args_t a;
    gpl_args_defaults(&a);
    a.op = (gpl_op_t)op;
    a.size = size;
    return gpl_workload_bytes_per_iter(&a);
}

// The reference's powervirus kernel itself, for power comparisons on the
// same box: one launch with the reference's grid (4 x SMs) and `inner`.
int ref_powervirus_launch(const unsigned char *d_role, const float4 *d_stream, size_t stream_elems,
                          int inner, float *d_sink, int blocks, size_t shmem, cudaStream_t stream) {
    gpl_powervirus_kernel<<<blocks, GPL_BLOCK_DIM, shmem, stream>>>(d_role, d_stream, stream_elems,
                                                                    inner, d_sink);
    return (int)cudaGetLastError();
}

int ref_pv_block_dim(void) { return GPL_BLOCK_DIM; }

// The cuBLASLt wrapper (gemm_lt.h:17-43) through a heap-held handle, so the
// tests need not mirror the struct layout: allocate, then read the public
// device pointers dA, dB, dC, dD, dScaleA, dScaleB, dScaleD (in that order).
void *ref_lt_new(void) { return calloc(1, sizeof(gpl_lt_gemm_t)); }
void ref_lt_delete(void *g) { free(g); }
void ref_lt_ptrs(void *gv, void **out) {
    gpl_lt_gemm_t *g = (gpl_lt_gemm_t *)gv;
    out[0] = g->dA; out[1] = g->dB; out[2] = g->dC; out[3] = g->dD;
    out[4] = g->dScaleA; out[5] = g->dScaleB; out[6] = g->dScaleD;
}

// The powervirus rung's concurrent tensor stream (workload_powervirus.cu:
// 281-397) for one non-Lt precision, as the rung sets it up:
// tensor_stream_init allocates n x n A, B, C (0x3c fill; cuBLAS handle with
// CUBLAS_TENSOR_OP_MATH), the test seeds them through ref_ts_ptrs, and
// tensor_stream_enqueue issues `count` cublasGemmEx with beta = 1 (C += A*B).
struct RefTs {
    gpl_args_t args;
    gpl_workload_ctx_t ctx;
    gpl_tensor_stream_t ts;
};
void *ref_ts_new(int prec, int n) {
    RefTs *r = (RefTs *)calloc(1, sizeof(RefTs));
    gpl_args_defaults(&r->args);
    r->args.precision = (gpl_prec_t)prec;
    r->args.size = n;
    r->ctx.args = &r->args;
    if (tensor_stream_init(&r->ctx, &r->ts) != 0) {
        tensor_stream_free(&r->ts);
        free(r);
        return NULL;
    }
    return r;
}
void ref_ts_ptrs(void *rv, void **out) {
    RefTs *r = (RefTs *)rv;
    out[0] = r->ts.dA; out[1] = r->ts.dB; out[2] = r->ts.dC; out[3] = (void *)r->ts.stream;
}
void ref_ts_enqueue(void *rv, int count) { tensor_stream_enqueue(&((RefTs *)rv)->ts, count); }
void ref_ts_delete(void *rv) {
    RefTs *r = (RefTs *)rv;
    tensor_stream_free(&r->ts);
    free(r);
}

}  // extern "C"
