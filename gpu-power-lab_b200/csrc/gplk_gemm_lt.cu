// gplk_gemm_lt.cu - the runner's held-open GEMM handle (include/gemm_lt.h)
// on libgplk's tcgen05 GEMMs. Set-up allocates and seeds the operands once;
// gpl_lt_enqueue only launches, so per-call overhead stays out of the steady
// loop, as in runner/src/gemm_lt.cu.
//
// Sizes the kernels cannot take directly (TMA rows must be 16-byte multiples,
// so FP8 needs K % 16 == 0; the NVFP4 kernel needs K % 256 == 0) run on a
// padded copy: the public dA / dB (and dSFA / dSFB) keep the reference's
// n x n layout, and `workspace` holds K-padded copies whose pad is zero.
// Every enqueue first copies the operands in (2-D copies on g->stream), so a
// caller may rewrite dA / dB between enqueues as with the reference.
#include <cstdio>
#include <cstring>

#include "../../include/gemm_lt.h"
#include "gplk_ptx.cuh"

#define GPL_LT_ERR(fmt, ...) fprintf(stderr, "[runner][ERROR] gemm_lt: " fmt "\n", ##__VA_ARGS__)

namespace {

int lt_alloc(void** p, size_t bytes, const char* what) {
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
        GPL_LT_ERR("cuda malloc %s (%zu bytes): %s", what, bytes, cudaGetErrorString(e));
        *p = nullptr;
        return -1;
    }
    return 0;
}

void lt_release(gpl_lt_gemm_t* g) {
    void** bufs[] = {&g->dA, &g->dB, &g->dC, &g->dD, &g->dScaleA, &g->dScaleB, &g->dScaleD,
                     &g->dSFA, &g->dSFB, &g->dAlpha, &g->workspace};
    for (void** b : bufs) {
        if (*b) cudaFree(*b);
        *b = nullptr;
    }
}

const char* prec_label(gpl_prec_t p) {
    switch (p) {
        case GPL_PREC_FP8: return "fp8";
        case GPL_PREC_FP4: return "fp4";
        default: return "non-Lt";
    }
}

// K as the kernels see it: n rounded up to a multiple of 16 (FP8) or 256
// (NVFP4), so operand rows start on 16-byte boundaries and NVFP4 stages are
// whole.
int lt_padded_k(gpl_prec_t p, int n) {
    const int q = p == GPL_PREC_FP4 ? 256 : 16;
    return (n + q - 1) / q * q;
}

// Workspace layout of the padded path: A' | B' (n rows of Kp bytes, or Kp/2
// for NVFP4), then for NVFP4 SFA' | SFB' in the K = Kp scale layout.
size_t lt_row_bytes(gpl_prec_t p, int k) { return p == GPL_PREC_FP4 ? (size_t)k / 2 : (size_t)k; }
size_t lt_padded_bytes(gpl_prec_t p, int n) {
    const int kp = lt_padded_k(p, n);
    size_t b = 2 * (size_t)n * lt_row_bytes(p, kp);
    if (p == GPL_PREC_FP4) b += 2 * gplk_nvfp4_sf_bytes(n, kp);
    return b;
}

// Copies the public n x n operands into the padded workspace on g->stream.
int lt_refresh_padded(gpl_lt_gemm_t* g) {
    const int n = g->n, kp = lt_padded_k(g->prec, n);
    const size_t src_row = lt_row_bytes(g->prec, n), dst_row = lt_row_bytes(g->prec, kp);
    uint8_t* ap = static_cast<uint8_t*>(g->workspace);
    uint8_t* bp = ap + (size_t)n * dst_row;
    if (cudaMemcpy2DAsync(ap, dst_row, g->dA, src_row, src_row, (size_t)n, cudaMemcpyDeviceToDevice, g->stream) !=
            cudaSuccess ||
        cudaMemcpy2DAsync(bp, dst_row, g->dB, src_row, src_row, (size_t)n, cudaMemcpyDeviceToDevice, g->stream) !=
            cudaSuccess)
        return -1;
    if (g->prec == GPL_PREC_FP4) {
        // Scale blocks of 512 bytes: (r/128, kb/4) at ((r/128) * kb4 + kb/4) * 512,
        // so each 128-row group is one contiguous run of kb4 blocks.
        const size_t kb4 = ((size_t)(n / 16) + 3) / 4, kb4p = ((size_t)(kp / 16) + 3) / 4;
        const size_t groups = ((size_t)n + 127) / 128;
        uint8_t* sfa = bp + (size_t)n * dst_row;
        uint8_t* sfb = sfa + gplk_nvfp4_sf_bytes(n, kp);
        if (cudaMemcpy2DAsync(sfa, kb4p * 512, g->dSFA, kb4 * 512, kb4 * 512, groups, cudaMemcpyDeviceToDevice,
                              g->stream) != cudaSuccess ||
            cudaMemcpy2DAsync(sfb, kb4p * 512, g->dSFB, kb4 * 512, kb4 * 512, groups, cudaMemcpyDeviceToDevice,
                              g->stream) != cudaSuccess)
            return -1;
    }
    return 0;
}

}  // namespace

extern "C" bool gpl_lt_precision_supported(gpl_prec_t p) {
    if (p != GPL_PREC_FP8 && p != GPL_PREC_FP4) return false;
    gplk::DeviceInfo d;
    return gplk::require_sm100(&d) == GPLK_STATUS_OK;
}

extern "C" int gpl_lt_init(gpl_lt_gemm_t* g, gpl_prec_t prec, int n, cudaStream_t stream) {
    memset(g, 0, sizeof(*g));
    g->n = n;
    g->prec = prec;
    g->stream = stream;
    if (prec != GPL_PREC_FP8 && prec != GPL_PREC_FP4) {
        GPL_LT_ERR("precision %d is not an Lt format", (int)prec);
        return -1;
    }
    gplk::DeviceInfo d;
    if (gplk::require_sm100(&d) != GPLK_STATUS_OK) {
        GPL_LT_ERR("no %s algorithm available on this device (needs sm_100)", prec_label(prec));
        return -1;
    }
    if (n <= 0 || (prec == GPL_PREC_FP4 && n % 32 != 0)) {
        GPL_LT_ERR("n=%d unsupported for %s (%s)", n, prec_label(prec),
                   prec == GPL_PREC_FP4 ? "a multiple of 32 is required: rows of n/2 bytes on 16-byte boundaries"
                                        : "n must be positive");
        return -1;
    }
    const size_t nn = (size_t)n * (size_t)n;
    const size_t ab_bytes = prec == GPL_PREC_FP8 ? nn : nn / 2;
    const size_t cd_bytes = nn * 2;
    const float one = 1.0f;
    if (lt_alloc(&g->dA, ab_bytes, "A") || lt_alloc(&g->dB, ab_bytes, "B") || lt_alloc(&g->dC, cd_bytes, "C") ||
        lt_alloc(&g->dD, cd_bytes, "D") || lt_alloc(&g->dScaleA, 4, "scaleA") ||
        lt_alloc(&g->dScaleB, 4, "scaleB") || lt_alloc(&g->dScaleD, 4, "scaleD") ||
        lt_alloc(&g->dAlpha, 4, "alpha")) {
        lt_release(g);
        return -1;
    }
    // 0x38 is E4M3 1.0 (and the FP4 pair -0 / 1.5): unremarkable values, as
    // in the reference. Scales 1.0.
    bool ok = cudaMemset(g->dA, 0x38, ab_bytes) == cudaSuccess && cudaMemset(g->dB, 0x38, ab_bytes) == cudaSuccess &&
              cudaMemset(g->dC, 0, cd_bytes) == cudaSuccess &&
              cudaMemcpy(g->dScaleA, &one, 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(g->dScaleB, &one, 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(g->dScaleD, &one, 4, cudaMemcpyHostToDevice) == cudaSuccess &&
              cudaMemcpy(g->dAlpha, &one, 4, cudaMemcpyHostToDevice) == cudaSuccess;
    if (ok && prec == GPL_PREC_FP4) {
        const size_t sf = gplk_nvfp4_sf_bytes(n, n);
        if (lt_alloc(&g->dSFA, sf, "SFA") || lt_alloc(&g->dSFB, sf, "SFB")) {
            lt_release(g);
            return -1;
        }
        ok = cudaMemset(g->dSFA, 0x38, sf) == cudaSuccess && cudaMemset(g->dSFB, 0x38, sf) == cudaSuccess;
    }
    if (ok && lt_padded_k(prec, n) != n) {
        // K-padded operand copies (zero pad), refreshed by every enqueue.
        g->workspace_bytes = lt_padded_bytes(prec, n);
        if (lt_alloc(&g->workspace, g->workspace_bytes, "padded operands")) {
            lt_release(g);
            return -1;
        }
        ok = cudaMemset(g->workspace, 0, g->workspace_bytes) == cudaSuccess;
    }
    if (!ok) {
        GPL_LT_ERR("initialising %s operands failed: %s", prec_label(prec), cudaGetErrorString(cudaGetLastError()));
        lt_release(g);
        return -1;
    }
    g->ready = true;
    if (g->workspace)
        fprintf(stderr, "[runner] gemm_lt: %s GEMM n=%d ready (tcgen05, K padded to %d in a %zu-byte workspace)\n",
                prec_label(prec), n, lt_padded_k(prec, n), g->workspace_bytes);
    else
        fprintf(stderr, "[runner] gemm_lt: %s GEMM n=%d ready (tcgen05, no workspace)\n", prec_label(prec), n);
    return 0;
}

extern "C" int gpl_lt_enqueue(gpl_lt_gemm_t* g, int count) {
    if (!g->ready) return -1;
    const int n = g->n, kp = lt_padded_k(g->prec, n);
    const uint8_t *A = (const uint8_t*)g->dA, *B = (const uint8_t*)g->dB;
    const uint8_t *SFA = (const uint8_t*)g->dSFA, *SFB = (const uint8_t*)g->dSFB;
    if (kp != n) {
        const size_t row = lt_row_bytes(g->prec, kp);
        A = static_cast<const uint8_t*>(g->workspace);
        B = A + (size_t)n * row;
        SFA = B + (size_t)n * row;
        SFB = SFA + (g->prec == GPL_PREC_FP4 ? gplk_nvfp4_sf_bytes(n, kp) : 0);
    }
    if (count > 0 && kp != n && lt_refresh_padded(g) != 0) {
        GPL_LT_ERR("%s operand copy failed: %s", prec_label(g->prec), cudaGetErrorString(cudaGetLastError()));
        return -1;
    }
    for (int i = 0; i < count; ++i) {
        int st;
        if (g->prec == GPL_PREC_FP8) {
            st = gplk_gemm_fp8_tn(A, B, (uint16_t*)g->dD, n, n, kp, (const float*)g->dScaleA,
                                  (const float*)g->dScaleB, g->stream);
        } else {
            st = gplk_gemm_nvfp4_tn(A, B, SFA, SFB, (uint16_t*)g->dD, n, n, kp, (const float*)g->dAlpha, g->stream);
        }
        if (st != GPLK_STATUS_OK) {
            GPL_LT_ERR("%s GEMM launch failed: %s", prec_label(g->prec), gplk_status_string(st));
            return -1;
        }
    }
    return 0;
}

extern "C" void gpl_lt_free(gpl_lt_gemm_t* g) {
    if (!g->ready) return;
    lt_release(g);
    g->ready = false;
}
