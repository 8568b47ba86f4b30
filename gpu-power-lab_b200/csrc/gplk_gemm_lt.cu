// gplk_gemm_lt.cu - the runner's held-open GEMM handle (include/gemm_lt.h)
// on libgplk's tcgen05 GEMMs. Set-up allocates and seeds the operands once;
// gpl_lt_enqueue only launches, so per-call overhead stays out of the steady
// loop, as in runner/src/gemm_lt.cu.
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
    if (n <= 0 || n % 16 != 0 || (prec == GPL_PREC_FP4 && n % 256 != 0)) {
        GPL_LT_ERR("n=%d unsupported for %s (multiple of %d required)", n, prec_label(prec),
                   prec == GPL_PREC_FP4 ? 256 : 16);
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
    if (!ok) {
        GPL_LT_ERR("initialising %s operands failed: %s", prec_label(prec), cudaGetErrorString(cudaGetLastError()));
        lt_release(g);
        return -1;
    }
    g->ready = true;
    fprintf(stderr, "[runner] gemm_lt: %s GEMM n=%d ready (tcgen05, no workspace)\n", prec_label(prec), n);
    return 0;
}

extern "C" int gpl_lt_enqueue(gpl_lt_gemm_t* g, int count) {
    if (!g->ready) return -1;
    const int n = g->n;
    for (int i = 0; i < count; ++i) {
        int st;
        if (g->prec == GPL_PREC_FP8) {
            st = gplk_gemm_fp8_tn((const uint8_t*)g->dA, (const uint8_t*)g->dB, (uint16_t*)g->dD, n, n, n,
                                  (const float*)g->dScaleA, (const float*)g->dScaleB, g->stream);
        } else {
            st = gplk_gemm_nvfp4_tn((const uint8_t*)g->dA, (const uint8_t*)g->dB, (const uint8_t*)g->dSFA,
                                    (const uint8_t*)g->dSFB, (uint16_t*)g->dD, n, n, n, (const float*)g->dAlpha,
                                    g->stream);
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
