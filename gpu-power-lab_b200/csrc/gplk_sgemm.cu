// gplk_sgemm.cu - true-FP32 SIMT SGEMM (FFMA, no TF32), row-major.
//
// Register-blocked tiles: a CTA computes BM x BN of C, each thread TM x TN
// split into two halves along each dimension (rows ty*TM/2 and BM/2 +
// ty*TM/2, likewise for columns) so shared-memory reads of a warp are either
// broadcasts or contiguous 128-bit loads. K is walked in BK slices through
// a double-buffered shared-memory ring; the next slice is fetched into
// registers while the current one is multiplied.
// Each output is one FP32 FFMA chain over k = 0..K-1 in order, so the result
// differs from a double-accumulated host loop only by FP32 rounding.
#include "gplk_ptx.cuh"

namespace gplk {
namespace sgemm {

// W consecutive floats from shared memory (16-byte aligned for W % 4 == 0,
// 8-byte aligned for W == 2).
template <int W>
__device__ __forceinline__ void lds_vec(const float* p, float* out) {
    if constexpr (W % 4 == 0) {
#pragma unroll
        for (int i = 0; i < W; i += 4) {
            const float4 v = *reinterpret_cast<const float4*>(p + i);
            out[i] = v.x, out[i + 1] = v.y, out[i + 2] = v.z, out[i + 3] = v.w;
        }
    } else if constexpr (W == 2) {
        const float2 v = *reinterpret_cast<const float2*>(p);
        out[0] = v.x, out[1] = v.y;
    } else {
#pragma unroll
        for (int i = 0; i < W; ++i) out[i] = p[i];
    }
}

template <int W>
__device__ __forceinline__ void stg_vec(float* p, const float* v) {
    if constexpr (W % 4 == 0) {
#pragma unroll
        for (int j = 0; j < W; j += 4)
            *reinterpret_cast<float4*>(p + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else if constexpr (W == 2) {
        *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    } else {
#pragma unroll
        for (int j = 0; j < W; ++j) p[j] = v[j];
    }
}

template <int BM, int BN, int BK, int TM, int TN, bool VEC>
struct Cfg {
    static constexpr int kThreads = (BM / TM) * (BN / TN);
    static constexpr int kApad = 4;  // keeps transposed A stores off one bank
    static constexpr int kALoads = BM * BK / 4 / kThreads;  // float4 per thread
    static constexpr int kBLoads = BK * BN / 4 / kThreads;
    static_assert(BM * BK % (4 * kThreads) == 0, "A tile split");
    static_assert(BK * BN % (4 * kThreads) == 0, "B tile split");
};

template <int BM, int BN, int BK, int TM, int TN, bool VEC>
__global__ void __launch_bounds__(Cfg<BM, BN, BK, TM, TN, VEC>::kThreads)
    sgemm_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C,
                 int M, int N, int K, int lda, int ldb, int ldc) {
    using CF = Cfg<BM, BN, BK, TM, TN, VEC>;
    constexpr int T = CF::kThreads;
    constexpr int TM2 = TM / 2, TN2 = TN / 2;
    __shared__ __align__(16) float As[2][BK][BM + CF::kApad];
    __shared__ __align__(16) float Bs[2][BK][BN];

    const int tid = threadIdx.x;
    const int tx = tid % (BN / TN);
    const int ty = tid / (BN / TN);
    const int m0 = blockIdx.y * BM;
    const int n0 = blockIdx.x * BN;

    float4 ra[CF::kALoads], rb[CF::kBLoads];

    // A slice: BM rows x BK columns, as float4 along K.
    auto load_a = [&](int k0) {
#pragma unroll
        for (int i = 0; i < CF::kALoads; ++i) {
            const int idx = tid + i * T;
            const int r = idx / (BK / 4), c4 = idx % (BK / 4);
            const int gm = m0 + r, gk = k0 + c4 * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (VEC) {
                if (gm < M && gk < K) v = *reinterpret_cast<const float4*>(A + (size_t)gm * lda + gk);
            } else {
                const float* p = A + (size_t)gm * lda + gk;
                if (gm < M) {
                    if (gk + 0 < K) v.x = p[0];
                    if (gk + 1 < K) v.y = p[1];
                    if (gk + 2 < K) v.z = p[2];
                    if (gk + 3 < K) v.w = p[3];
                }
            }
            ra[i] = v;
        }
    };
    auto load_b = [&](int k0) {
#pragma unroll
        for (int i = 0; i < CF::kBLoads; ++i) {
            const int idx = tid + i * T;
            const int r = idx / (BN / 4), c4 = idx % (BN / 4);
            const int gk = k0 + r, gn = n0 + c4 * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (VEC) {
                if (gk < K && gn < N) v = *reinterpret_cast<const float4*>(B + (size_t)gk * ldb + gn);
            } else {
                const float* p = B + (size_t)gk * ldb + gn;
                if (gk < K) {
                    if (gn + 0 < N) v.x = p[0];
                    if (gn + 1 < N) v.y = p[1];
                    if (gn + 2 < N) v.z = p[2];
                    if (gn + 3 < N) v.w = p[3];
                }
            }
            rb[i] = v;
        }
    };
    auto store_tiles = [&](int buf) {
#pragma unroll
        for (int i = 0; i < CF::kALoads; ++i) {
            const int idx = tid + i * T;
            const int r = idx / (BK / 4), c4 = idx % (BK / 4);
            As[buf][c4 * 4 + 0][r] = ra[i].x;
            As[buf][c4 * 4 + 1][r] = ra[i].y;
            As[buf][c4 * 4 + 2][r] = ra[i].z;
            As[buf][c4 * 4 + 3][r] = ra[i].w;
        }
#pragma unroll
        for (int i = 0; i < CF::kBLoads; ++i) {
            const int idx = tid + i * T;
            const int r = idx / (BN / 4), c4 = idx % (BN / 4);
            *reinterpret_cast<float4*>(&Bs[buf][r][c4 * 4]) = rb[i];
        }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

    const int ktiles = (K + BK - 1) / BK;
    load_a(0);
    load_b(0);
    store_tiles(0);
    __syncthreads();

    for (int kt = 0; kt < ktiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < ktiles) {
            load_a((kt + 1) * BK);
            load_b((kt + 1) * BK);
        }
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            float a[TM], b[TN];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                lds_vec<TM2>(&As[buf][k][h * (BM / 2) + ty * TM2], &a[h * TM2]);
                lds_vec<TN2>(&Bs[buf][k][h * (BN / 2) + tx * TN2], &b[h * TN2]);
            }
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
        if (kt + 1 < ktiles) {
            store_tiles(buf ^ 1);
        }
        __syncthreads();
    }

    // Epilogue: rows (h, i) and column groups (g, j) as in the k-loop.
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int i = 0; i < TM2; ++i) {
            const int gm = m0 + h * (BM / 2) + ty * TM2 + i;
            if (gm >= M) continue;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                const int gn = n0 + g * (BN / 2) + tx * TN2;
                float* crow = C + (size_t)gm * ldc + gn;
                const float* v = &acc[h * TM2 + i][g * TN2];
                if (VEC && gn + TN2 <= N) {
                    stg_vec<TN2>(crow, v);
                } else {
#pragma unroll
                    for (int j = 0; j < TN2; ++j)
                        if (gn + j < N) crow[j] = v[j];
                }
            }
        }
    }
}

template <int BM, int BN, int BK, int TM, int TN>
static int launch(const float* A, const float* B, float* C, int M, int N, int K, int lda, int ldb,
                  int ldc, bool vec, cudaStream_t stream) {
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    if (vec) {
        sgemm_kernel<BM, BN, BK, TM, TN, true>
            <<<grid, Cfg<BM, BN, BK, TM, TN, true>::kThreads, 0, stream>>>(A, B, C, M, N, K, lda, ldb, ldc);
    } else {
        sgemm_kernel<BM, BN, BK, TM, TN, false>
            <<<grid, Cfg<BM, BN, BK, TM, TN, false>::kThreads, 0, stream>>>(A, B, C, M, N, K, lda, ldb, ldc);
    }
    return launch_status(cudaGetLastError());
}

}  // namespace sgemm
}  // namespace gplk

extern "C" int gplk_sgemm_f32(const float* A, const float* B, float* C, int M, int N, int K, int lda,
                              int ldb, int ldc, cudaStream_t stream) {
    using namespace gplk;
    if (M < 0 || N < 0 || K < 0) return GPLK_STATUS_BAD_ARG;
    if (M == 0 || N == 0) return GPLK_STATUS_OK;
    if (!C || (K > 0 && (!A || !B))) return GPLK_STATUS_BAD_ARG;  // K == 0: A, B unread
    if ((K > 0 && (lda < K || ldb < N)) || ldc < N) return GPLK_STATUS_BAD_ARG;
    DeviceInfo d;
    int st = current_device_info(&d);
    if (st != GPLK_STATUS_OK) return st;
    const bool vec = aligned16(A) && aligned16(B) && aligned16(C) && (lda % 4 == 0) && (ldb % 4 == 0) &&
                     (ldc % 4 == 0) && (K % 4 == 0) && (N % 4 == 0);
    // Large problems: 128 x 128 tiles (8 x 8 per thread). When that leaves
    // SMs idle, 64 x 64 tiles (4 x 4 per thread) give more CTAs to spread.
    const long tiles128 = (long)((M + 127) / 128) * ((N + 127) / 128);
    if (tiles128 >= 2L * d.sm_count)
        return sgemm::launch<128, 128, 16, 8, 8>(A, B, C, M, N, K, lda, ldb, ldc, vec, stream);
    return sgemm::launch<64, 64, 16, 4, 4>(A, B, C, M, N, K, lda, ldb, ldc, vec, stream);
}
