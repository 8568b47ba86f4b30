/*
 * workload_util.c - work accounting that feeds the summary's TFLOPS and
 * GB/s (drop-in for the runner's workload_util.c, same formulae at
 * runner/src/workload_util.c:20-58, plus the powervirus tensor-stream case).
 *
 *   sgemm (any precision, now including fp8 and fp4): 2 N^3 per GEMM
 *   powervirus with --tensor-backend cublas and no kernel (tensor-only):
 *       mix_tensor / streams N^3 GEMMs per iteration on the tensor stream
 *       (the reference reported 0 TFLOPS for these rungs)
 *   memstream: 3 arrays x size^2 x 4 B
 *   fft: 2 x size x batch x 8 B, batch = max(1, 2^20 / size)
 */
#include "workload.h"

double gpl_workload_flops_per_iter(const gpl_args_t *a) {
    const double n = (double)a->size;
    switch (a->op) {
        case GPL_OP_SGEMM:
            return 2.0 * n * n * n;
        case GPL_OP_POWERVIRUS:
            /* mix_tensor GEMMs per `streams` kernel iterations, as the
             * driver enqueues them (workload_powervirus.cu here and in the
             * reference, :603-657). */
            if (a->tensor_cublas && a->mix_tensor > 0 && a->mix_fma == 0 && a->mix_dram == 0)
                return 2.0 * n * n * n * (double)a->mix_tensor / (double)(a->streams > 0 ? a->streams : 1);
            return 0.0;
        default:
            return 0.0;
    }
}

double gpl_workload_bytes_per_iter(const gpl_args_t *a) {
    switch (a->op) {
        case GPL_OP_MEMSTREAM: {
            const double n = (double)a->size;
            return 3.0 * n * n * 4.0;
        }
        case GPL_OP_FFT: {
            int batch = (1 << 20) / a->size;
            if (batch < 1) batch = 1;
            return 2.0 * (double)a->size * (double)batch * 8.0;
        }
        default:
            return 0.0;
    }
}
