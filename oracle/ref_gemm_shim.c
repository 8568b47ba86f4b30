/* ref_gemm_shim.c - the reference runner's cublasGemmEx GEMM rung, compiled
 * from its own source (ref_build.sh), as a GPU checker for libgplk's dense
 * tensor-core GEMMs. TEST INFRASTRUCTURE ONLY: the parity tests call it,
 * the product never does.
 *
 * runner/src/workload_gemm.c keeps its precision -> cuBLAS type mapping
 * (prec_to_cublas, :44-79) `static`, so this file includes the source
 * textually and wraps one GEMM exactly as the rung issues it: the math mode
 * of :127-132, the host scalars of :137-153 and the call of :155-163
 * (CUBLAS_OP_N twice, n x n x n, every leading dimension n,
 * CUBLAS_GEMM_DEFAULT_TENSOR_OP).
 */
#include "workload_gemm.c"

/* One column-major C = A * B of the rung's precision `prec` (gpl_prec_t) on
 * `stream`. Returns the cublasStatus_t of the call (0 = success). */
int ref_gemm_ex(int prec, const void *A, const void *B, void *C, int n, cudaStream_t stream) {
    static cublasHandle_t h = NULL;
    if (!h && cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) return -1;
    cudaDataType inT, outT;
    cublasComputeType_t cT;
    prec_to_cublas((gpl_prec_t)prec, &inT, &outT, &cT);
    cublasSetStream(h, stream);
    cublasSetMathMode(h, prec == GPL_PREC_TF32 ? CUBLAS_TF32_TENSOR_OP_MATH : CUBLAS_DEFAULT_MATH);
    float alpha_f = 1.0f, beta_f = 0.0f;
    unsigned short alpha_h = 0x3C00, beta_h = 0x0000;
    double alpha_d = 1.0, beta_d = 0.0;
    int alpha_i = 1, beta_i = 0;
    const void *alpha_p = &alpha_f, *beta_p = &beta_f;
    if (cT == CUBLAS_COMPUTE_16F) { alpha_p = &alpha_h; beta_p = &beta_h; }
    else if (cT == CUBLAS_COMPUTE_64F) { alpha_p = &alpha_d; beta_p = &beta_d; }
    else if (cT == CUBLAS_COMPUTE_32I) { alpha_p = &alpha_i; beta_p = &beta_i; }
    return (int)cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, n, n, n, alpha_p, A, inT, n, B, inT, n, beta_p, C, outT, n,
                             cT, CUBLAS_GEMM_DEFAULT_TENSOR_OP);
}
