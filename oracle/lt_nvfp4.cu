// lt_nvfp4.cu - cuBLASLt NVFP4 GEMM harness: the library path the reference's
// gemm_lt.cu (runner/src/gemm_lt.cu:76-82, GPL_PREC_FP4) aims at, configured
// with the block scales that path omits. TEST INFRASTRUCTURE ONLY: the parity
// tests call it as the checker for libgplk's NVFP4 GEMM.
//
// Same descriptor shape as the reference's FP8 path (TRANSA=T, TRANSB=N,
// n x n layouts with ld = K, FP32 compute and scale type, BF16 C/D, 32 MiB
// workspace, first heuristic), plus
//   CUBLASLT_MATMUL_DESC_{A,B}_SCALE_MODE = VEC16_UE4M3,
//   CUBLASLT_MATMUL_DESC_{A,B}_SCALE_POINTER = the block-scale arrays,
//   alpha = product of the per-tensor global scales.
#include <cublasLt.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#define LT(x)                                                              \
    do {                                                                   \
        cublasStatus_t _s = (x);                                           \
        if (_s != CUBLAS_STATUS_SUCCESS) {                                 \
            fprintf(stderr, "lt_nvfp4: %s -> %d\n", #x, (int)_s);          \
            rc = (int)_s;                                                  \
            goto done;                                                     \
        }                                                                  \
    } while (0)

extern "C" int oracle_lt_gemm_nvfp4_tn(const void *A, const void *B, const void *SFA, const void *SFB,
                                       void *D, int M, int N, int K, float alpha, void *workspace,
                                       size_t workspace_bytes, cudaStream_t stream) {
    int rc = 0;
    cublasLtHandle_t lt = nullptr;
    cublasLtMatmulDesc_t op = nullptr;
    cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr, ld = nullptr;
    cublasLtMatmulPreference_t pref = nullptr;
    cublasLtMatmulHeuristicResult_t heur;
    int returned = 0;
    const float beta = 0.0f;
    cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
    cublasLtMatmulMatrixScale_t mode = CUBLASLT_MATMUL_MATRIX_SCALE_VEC16_UE4M3;

    LT(cublasLtCreate(&lt));
    LT(cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta)));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb)));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_A_SCALE_MODE, &mode, sizeof(mode)));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_B_SCALE_MODE, &mode, sizeof(mode)));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_A_SCALE_POINTER, &SFA, sizeof(SFA)));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_B_SCALE_POINTER, &SFB, sizeof(SFB)));
    // A is K x M column-major (transposed to M x K), B is K x N, D is M x N.
    LT(cublasLtMatrixLayoutCreate(&la, CUDA_R_4F_E2M1, K, M, K));
    LT(cublasLtMatrixLayoutCreate(&lb, CUDA_R_4F_E2M1, K, N, K));
    LT(cublasLtMatrixLayoutCreate(&lc, CUDA_R_16BF, M, N, M));
    LT(cublasLtMatrixLayoutCreate(&ld, CUDA_R_16BF, M, N, M));
    LT(cublasLtMatmulPreferenceCreate(&pref));
    LT(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES,
                                            &workspace_bytes, sizeof(workspace_bytes)));
    LT(cublasLtMatmulAlgoGetHeuristic(lt, op, la, lb, lc, ld, pref, 1, &heur, &returned));
    if (returned == 0) {
        fprintf(stderr, "lt_nvfp4: no algorithm\n");
        rc = -1;
        goto done;
    }
    LT(cublasLtMatmul(lt, op, &alpha, A, la, B, lb, &beta, D, lc, D, ld, &heur.algo, workspace,
                      workspace_bytes, stream));
done:
    if (pref) cublasLtMatmulPreferenceDestroy(pref);
    if (ld) cublasLtMatrixLayoutDestroy(ld);
    if (lc) cublasLtMatrixLayoutDestroy(lc);
    if (lb) cublasLtMatrixLayoutDestroy(lb);
    if (la) cublasLtMatrixLayoutDestroy(la);
    if (op) cublasLtMatmulDescDestroy(op);
    if (lt) cublasLtDestroy(lt);
    return rc;
}

// The same call repeated `count` times on one set of descriptors, for the
// library-throughput comparison (cuBLASLt is the bar the reference sets).
extern "C" int oracle_lt_gemm_nvfp4_tn_timed(const void *A, const void *B, const void *SFA,
                                             const void *SFB, void *D, int M, int N, int K, float alpha,
                                             void *workspace, size_t workspace_bytes, int count,
                                             cudaStream_t stream, float *ms_out) {
    int rc = 0;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cublasLtHandle_t lt = nullptr;
    cublasLtMatmulDesc_t op = nullptr;
    cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr, ld = nullptr;
    cublasLtMatmulPreference_t pref = nullptr;
    cublasLtMatmulHeuristicResult_t heur;
    int returned = 0;
    const float beta = 0.0f;
    cublasOperation_t ta = CUBLAS_OP_T, tb = CUBLAS_OP_N;
    cublasLtMatmulMatrixScale_t mode = CUBLASLT_MATMUL_MATRIX_SCALE_VEC16_UE4M3;
    LT(cublasLtCreate(&lt));
    LT(cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSA, &ta, sizeof(ta)));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_TRANSB, &tb, sizeof(tb)));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_A_SCALE_MODE, &mode, sizeof(mode)));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_B_SCALE_MODE, &mode, sizeof(mode)));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_A_SCALE_POINTER, &SFA, sizeof(SFA)));
    LT(cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_B_SCALE_POINTER, &SFB, sizeof(SFB)));
    LT(cublasLtMatrixLayoutCreate(&la, CUDA_R_4F_E2M1, K, M, K));
    LT(cublasLtMatrixLayoutCreate(&lb, CUDA_R_4F_E2M1, K, N, K));
    LT(cublasLtMatrixLayoutCreate(&lc, CUDA_R_16BF, M, N, M));
    LT(cublasLtMatrixLayoutCreate(&ld, CUDA_R_16BF, M, N, M));
    LT(cublasLtMatmulPreferenceCreate(&pref));
    LT(cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES,
                                            &workspace_bytes, sizeof(workspace_bytes)));
    LT(cublasLtMatmulAlgoGetHeuristic(lt, op, la, lb, lc, ld, pref, 1, &heur, &returned));
    if (returned == 0) { rc = -1; goto done; }
    for (int i = 0; i < 2; ++i)
        LT(cublasLtMatmul(lt, op, &alpha, A, la, B, lb, &beta, D, lc, D, ld, &heur.algo, workspace,
                          workspace_bytes, stream));
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, stream);
    for (int i = 0; i < count; ++i)
        LT(cublasLtMatmul(lt, op, &alpha, A, la, B, lb, &beta, D, lc, D, ld, &heur.algo, workspace,
                          workspace_bytes, stream));
    cudaEventRecord(e1, stream);
    cudaEventSynchronize(e1);
    cudaEventElapsedTime(ms_out, e0, e1);
done:
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (pref) cublasLtMatmulPreferenceDestroy(pref);
    if (ld) cublasLtMatrixLayoutDestroy(ld);
    if (lc) cublasLtMatrixLayoutDestroy(lc);
    if (lb) cublasLtMatrixLayoutDestroy(lb);
    if (la) cublasLtMatrixLayoutDestroy(la);
    if (op) cublasLtMatmulDescDestroy(op);
    if (lt) cublasLtDestroy(lt);
    return rc;
}
