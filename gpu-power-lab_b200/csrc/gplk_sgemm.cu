// gplk_sgemm.cu - true-FP32 SIMT SGEMM (FFMA, no TF32), row-major.
//
// Three kernel families, chosen by gplk_sgemm_f32 at the end of the file:
//   * 16-byte-aligned operands (the runner's case): the cp.async + paired
//     FFMA main loop (sgemm_v2_kernel, 128 x 128 tiles, 8 x 16 outputs per
//     thread), or, when the tiles leave the last wave of SMs ragged,
//     stream-K over one block per SM (sgemm_sk_kernel, 8 x 8 per thread);
//   * anything else: the register-staged kernels below (sgemm_kernel, and a
//     2-CTA cluster split of K for problems with few tiles).
// The register-staged kernels: a CTA computes BM x BN of C, each thread
// TM x TN split into two halves along each dimension (rows ty*TM/2 and
// BM/2 + ty*TM/2, likewise for columns) so shared-memory reads of a warp are
// either broadcasts or contiguous 128-bit loads. K is walked in BK slices
// through a double-buffered shared-memory ring; the next slice is fetched
// into registers while the current one is multiplied.
// Each output is one FP32 FFMA chain over k in order (split-K and stream-K
// add a few such chains in a fixed order), so the result differs from a
// double-accumulated host loop only by FP32 rounding.
#include <mutex>
#include <vector>

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

// C = acc + beta * C_old for the W values at p (beta != 0: the old values
// are read first; fmaf(beta, old, acc) is acc + old exactly rounded once for
// beta = 1, as cuBLAS computes alpha * acc + beta * C with alpha = 1).
template <int W>
__device__ __forceinline__ void add_old_vec(const float* p, float beta, float* v) {
    if constexpr (W % 4 == 0) {
#pragma unroll
        for (int j = 0; j < W; j += 4) {
            const float4 o = __ldcs(reinterpret_cast<const float4*>(p + j));
            v[j] = __fmaf_rn(beta, o.x, v[j]);
            v[j + 1] = __fmaf_rn(beta, o.y, v[j + 1]);
            v[j + 2] = __fmaf_rn(beta, o.z, v[j + 2]);
            v[j + 3] = __fmaf_rn(beta, o.w, v[j + 3]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < W; ++j) v[j] = __fmaf_rn(beta, p[j], v[j]);
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

// One BK slice of the register-blocked product: acc[TM][TN] += A x B over
// k = 0..BK-1 in order. Fragments for k + 1 are read from shared memory
// while the FFMAs of k issue (register double buffering), so shared-memory
// latency hides behind arithmetic.
template <int BM, int BN, int BK, int TM, int TN, int APAD>
__device__ __forceinline__ void tile_fma(const float (*As)[BM + APAD], const float (*Bs)[BN], int tx, int ty,
                                         float (&acc)[TM][TN]) {
    constexpr int TM2 = TM / 2, TN2 = TN / 2;
    float a[2][TM], b[2][TN];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        lds_vec<TM2>(&As[0][h * (BM / 2) + ty * TM2], &a[0][h * TM2]);
        lds_vec<TN2>(&Bs[0][h * (BN / 2) + tx * TN2], &b[0][h * TN2]);
    }
#pragma unroll
    for (int k = 0; k < BK; ++k) {
        const int cur = k & 1;
        if (k + 1 < BK) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                lds_vec<TM2>(&As[k + 1][h * (BM / 2) + ty * TM2], &a[cur ^ 1][h * TM2]);
                lds_vec<TN2>(&Bs[k + 1][h * (BN / 2) + tx * TN2], &b[cur ^ 1][h * TN2]);
            }
        }
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(a[cur][i], b[cur][j], acc[i][j]);
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
                 int M, int N, int K, int lda, int ldb, int ldc, float beta) {
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
        tile_fma<BM, BN, BK, TM, TN, CF::kApad>(As[buf], Bs[buf], tx, ty, acc);
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
                float* v = &acc[h * TM2 + i][g * TN2];
                if (VEC && gn + TN2 <= N) {
                    if (beta != 0.f) add_old_vec<TN2>(crow, beta, v);
                    stg_vec<TN2>(crow, v);
                } else {
#pragma unroll
                    for (int j = 0; j < TN2; ++j)
                        if (gn + j < N) crow[j] = beta != 0.f ? __fmaf_rn(beta, crow[j], v[j]) : v[j];
                }
            }
        }
    }
}

// ------------------------------------------------------------ cluster split-K
// For problems with too few 128 x 128 tiles to fill the GPU, a 2-CTA cluster
// shares each tile: CTA r of the pair computes the partial product over its
// half of K, then CTA 1 writes its accumulators into CTA 0's shared memory
// (distributed shared memory, st.shared::cluster) and CTA 0 adds them to its
// own in a fixed order (own + peer) and stores C. Deterministic, and no
// global scratch, memset or atomics.
constexpr int kSplitThreads = 256;  // 128 x 128 tile, 8 x 8 per thread

template <bool VEC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kSplitThreads)
    sgemm_split2_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int M,
                        int N, int K, int lda, int ldb, int ldc, float beta) {
    constexpr int BM = 128, BN = 128, BK = 16, TM = 8, TN = 8;
    using CF = Cfg<BM, BN, BK, TM, TN, VEC>;
    constexpr int T = CF::kThreads;
    static_assert(T == kSplitThreads, "split tile threads");
    constexpr int TM2 = TM / 2, TN2 = TN / 2;
    extern __shared__ __align__(16) float split_smem[];
    float(*As)[BK][BM + CF::kApad] = reinterpret_cast<float(*)[BK][BM + CF::kApad]>(split_smem);
    float(*Bs)[BK][BN] = reinterpret_cast<float(*)[BK][BN]>(split_smem + 2 * BK * (BM + CF::kApad));
    float4* recv = reinterpret_cast<float4*>(split_smem + 2 * BK * (BM + CF::kApad) + 2 * BK * BN);  // [16][T]

    const uint32_t rank = cluster_ctarank();
    const int tid = threadIdx.x;
    const int tx = tid % (BN / TN);
    const int ty = tid / (BN / TN);
    const int m0 = blockIdx.y * BM;
    const int n0 = (blockIdx.x >> 1) * BN;
    // K range of this CTA: the first half (rounded to BK) for rank 0.
    const int k_half = ((K + 2 * BK - 1) / (2 * BK)) * BK;
    const int k_begin = rank == 0 ? 0 : k_half;
    const int k_end = rank == 0 ? min(K, k_half) : K;

    float4 ra[CF::kALoads], rb[CF::kBLoads];
    auto load_a = [&](int k0) {
#pragma unroll
        for (int i = 0; i < CF::kALoads; ++i) {
            const int idx = tid + i * T;
            const int r = idx / (BK / 4), c4 = idx % (BK / 4);
            const int gm = m0 + r, gk = k0 + c4 * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (VEC) {
                if (gm < M && gk < k_end) v = *reinterpret_cast<const float4*>(A + (size_t)gm * lda + gk);
            } else if (gm < M) {
                const float* q = A + (size_t)gm * lda + gk;
                if (gk + 0 < k_end) v.x = q[0];
                if (gk + 1 < k_end) v.y = q[1];
                if (gk + 2 < k_end) v.z = q[2];
                if (gk + 3 < k_end) v.w = q[3];
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
                if (gk < k_end && gn < N) v = *reinterpret_cast<const float4*>(B + (size_t)gk * ldb + gn);
            } else if (gk < k_end) {
                const float* q = B + (size_t)gk * ldb + gn;
                if (gn + 0 < N) v.x = q[0];
                if (gn + 1 < N) v.y = q[1];
                if (gn + 2 < N) v.z = q[2];
                if (gn + 3 < N) v.w = q[3];
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

    const int ktiles = k_end > k_begin ? (k_end - k_begin + BK - 1) / BK : 0;
    if (ktiles > 0) {
        load_a(k_begin);
        load_b(k_begin);
        store_tiles(0);
    }
    __syncthreads();
    for (int kt = 0; kt < ktiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < ktiles) {
            load_a(k_begin + (kt + 1) * BK);
            load_b(k_begin + (kt + 1) * BK);
        }
        tile_fma<BM, BN, BK, TM, TN, CF::kApad>(As[buf], Bs[buf], tx, ty, acc);
        if (kt + 1 < ktiles) store_tiles(buf ^ 1);
        __syncthreads();
    }

    // Hand-off: CTA 1 writes its 64 partial sums per thread into CTA 0's
    // receive buffer, laid out [v][thread] so each warp's float4 stores are
    // contiguous.
    if (rank == 1) {
        const uint32_t dst0 = mapa_shared(smem_u32(recv), 0);
#pragma unroll
        for (int v = 0; v < 16; ++v) {
            const int i = v / 2, j0 = (v % 2) * 4;
            const uint32_t addr = dst0 + (uint32_t)((v * T + tid) * 16);
            asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(acc[i][j0]),
                         "f"(acc[i][j0 + 1]), "f"(acc[i][j0 + 2]), "f"(acc[i][j0 + 3])
                         : "memory");
        }
    }
    cluster_sync();
    if (rank == 1) return;
#pragma unroll
    for (int v = 0; v < 16; ++v) {
        const int i = v / 2, j0 = (v % 2) * 4;
        const float4 q = recv[v * T + tid];
        acc[i][j0] = __fadd_rn(acc[i][j0], q.x);
        acc[i][j0 + 1] = __fadd_rn(acc[i][j0 + 1], q.y);
        acc[i][j0 + 2] = __fadd_rn(acc[i][j0 + 2], q.z);
        acc[i][j0 + 3] = __fadd_rn(acc[i][j0 + 3], q.w);
    }
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
                float* val = &acc[h * TM2 + i][g * TN2];
                if (VEC && gn + TN2 <= N) {
                    if (beta != 0.f) add_old_vec<TN2>(crow, beta, val);
                    stg_vec<TN2>(crow, val);
                } else {
#pragma unroll
                    for (int j = 0; j < TN2; ++j)
                        if (gn + j < N) crow[j] = beta != 0.f ? __fmaf_rn(beta, crow[j], val[j]) : val[j];
                }
            }
        }
    }
}

static int launch_split2(const float* A, const float* B, float* C, int M, int N, int K, int lda, int ldb, int ldc,
                         float beta, bool vec, cudaStream_t stream) {
    constexpr int BM = 128, BN = 128, BK = 16;
    const int smem = (int)(sizeof(float) * (2 * BK * (BM + 4) + 2 * BK * BN) + 16 * kSplitThreads * sizeof(float4));
    static thread_local uint64_t configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1ull << dev))) {
        if (cudaFuncSetAttribute(sgemm_split2_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
                cudaSuccess ||
            cudaFuncSetAttribute(sgemm_split2_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
                cudaSuccess)
            return GPLK_STATUS_LAUNCH_FAIL;
        configured |= 1ull << dev;
    }
    dim3 grid(2 * ((N + BN - 1) / BN), (M + BM - 1) / BM);
    if (vec)
        sgemm_split2_kernel<true><<<grid, kSplitThreads, smem, stream>>>(A, B, C, M, N, K, lda, ldb, ldc, beta);
    else
        sgemm_split2_kernel<false><<<grid, kSplitThreads, smem, stream>>>(A, B, C, M, N, K, lda, ldb, ldc, beta);
    return launch_status(cudaGetLastError());
}

// ------------------------------------------------------------ cp.async + FFMA2 main loop
// 128 x 128 tiles, 8 x 16 outputs per thread (128 threads) or 8 x 8 (256
// threads; layout in V2T below), BK = 16, a 3-stage ring filled
// by cp.async straight from global memory (no register staging). A stays
// K-major in shared memory (one 128-bit load = four k of one row), B stays
// N-major. The FFMAs issue as Blackwell's paired FP32 FMA (__ffma2_rn: two
// independent, individually rounded fmaf per instruction) on column pairs,
// halving the FMA issue slots. Each output is one FMA chain over k in order
// (or, under stream-K below, a fixed-order sum of a few such chains).
constexpr int kV2BM = 128, kV2BN = 128, kV2BK = 16, kV2Stages = 3;
// Thread layout for TN outputs per thread along N. Thread (tx, ty) owns rows
// ty + 16 i (i < 8) and TN / 4 groups of four columns, group h at
// h * GS + 4 tx. Both are conflict-free in shared memory: a warp's A reads
// hit rows of consecutive ty (80-byte pitch: distinct 16-byte bank groups)
// and its B reads cover 4 TX contiguous floats.
template <int TN>
struct V2T {
    static_assert(TN == 8 || TN == 16, "8 x 8 or 8 x 16 per thread");
    static constexpr int NP = TN / 2;           // column pairs per thread
    static constexpr int NG = TN / 4;           // column groups of four per thread
    static constexpr int TX = kV2BN / TN;       // threads along N
    static constexpr int GS = 4 * TX;           // column stride between a thread's groups
    static constexpr int Threads = TX * 16;     // 16 threads along M
    static constexpr int Park = 2 * TN;         // float4 per thread in a parked partial tile
};
// Whole-wave grids use 8 x 16 per thread (128 threads, two blocks per SM):
// 4096^3 measured 54.4 TFLOP/s against 50.3 with 8 x 8 (256 threads).
// Stream-K keeps 8 x 8: its extra state spills at 8 x 16, and with one
// block per SM 8 x 16 measured slower there (1024^3: 33.9 against 36.6).
constexpr int kV2TNDense = 16;
constexpr int kV2TNStreamK = 8;
constexpr int kV2APitch = kV2BK + 4;   // floats per A row in shared memory (80 B)
constexpr int kV2AStage = kV2BM * kV2APitch;
constexpr int kV2BStage = kV2BK * kV2BN;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const uint32_t dst = smem_u32(smem);
    const int src_bytes = valid ? 16 : 0;  // 0: fill the 16 bytes with zeros
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// acc += the 128 x 16 A slab x the 16 x 128 B slab of one ring stage.
template <int TN>
__device__ __forceinline__ void v2_ktile(const float* as, const float* bs, int tx, int ty,
                                         float2 (&acc)[8][TN / 2]) {
    using T = V2T<TN>;
#pragma unroll
    for (int kq = 0; kq < kV2BK; kq += 4) {
        float4 af[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            af[i] = *reinterpret_cast<const float4*>(as + (ty + 16 * i) * kV2APitch + kq);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            float2 bp[T::NP];
#pragma unroll
            for (int h = 0; h < T::NG; ++h) {
                const float4 b = *reinterpret_cast<const float4*>(bs + (kq + kk) * kV2BN + h * T::GS + tx * 4);
                bp[2 * h] = make_float2(b.x, b.y);
                bp[2 * h + 1] = make_float2(b.z, b.w);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float av = kk == 0 ? af[i].x : kk == 1 ? af[i].y : kk == 2 ? af[i].z : af[i].w;
                const float2 a2 = make_float2(av, av);
#pragma unroll
                for (int j = 0; j < T::NP; ++j) acc[i][j] = __ffma2_rn(a2, bp[j], acc[i][j]);
            }
        }
    }
}

// Copies one 16-wide K step of the 128 x 128 tile at (m0, n0) into a ring
// stage: 512 16-byte chunks of A (row r, k-quad q) and 512 of B spread over
// the threads; rows, columns and k past the matrix are zero-filled.
template <int TN>
__device__ __forceinline__ void v2_issue(const float* __restrict__ A, const float* __restrict__ B, int M, int N,
                                         int lda, int ldb, int m0, int n0, int k0, int k_end, float* as,
                                         float* bs) {
    constexpr int kThreads = V2T<TN>::Threads;
    const int tid = threadIdx.x;
#pragma unroll
    for (int i = 0; i < 512 / kThreads; ++i) {
        const int idx = tid + i * kThreads;  // 0..511
        const int r = idx >> 2, q = idx & 3;
        const int gm = m0 + r, gk = k0 + q * 4;
        const bool ok = gm < M && gk < k_end;
        cp_async16(as + r * kV2APitch + q * 4, ok ? A + (size_t)gm * lda + gk : A, ok);
    }
#pragma unroll
    for (int i = 0; i < 512 / kThreads; ++i) {
        const int idx = tid + i * kThreads;
        const int r = idx >> 5, c4 = idx & 31;
        const int gk = k0 + r, gn = n0 + c4 * 4;
        const bool ok = gk < k_end && gn < N;
        cp_async16(bs + r * kV2BN + c4 * 4, ok ? B + (size_t)gk * ldb + gn : B, ok);
    }
}

// The pipelined main loop: acc += A[m0.., k_begin..k_end) x B[k_begin..k_end, n0..]
// for one 128 x 128 tile, through the 3-stage cp.async ring in `smem`. On
// return every copy has landed and the block has synchronised, so the ring
// may be refilled for another tile.
template <int TN>
__device__ __forceinline__ void v2_mainloop(const float* __restrict__ A, const float* __restrict__ B, int M, int N,
                                            int lda, int ldb, int m0, int n0, int k_begin, int k_end,
                                            float* smem, float2 (&acc)[8][TN / 2]) {
    using T = V2T<TN>;
    float* As = smem;                          // [stage][128][kV2APitch]
    float* Bs = smem + kV2Stages * kV2AStage;  // [stage][16][128]
    const int tid = threadIdx.x;
    const int tx = tid % T::TX, ty = tid / T::TX;
    const int ktiles = k_end > k_begin ? (k_end - k_begin + kV2BK - 1) / kV2BK : 0;
    auto issue = [&](int kt) {
        const int st = kt % kV2Stages;
        v2_issue<TN>(A, B, M, N, lda, ldb, m0, n0, k_begin + kt * kV2BK, k_end, As + st * kV2AStage,
                 Bs + st * kV2BStage);
    };
#pragma unroll
    for (int s = 0; s < kV2Stages - 1; ++s) {
        if (s < ktiles) issue(s);
        cp_async_commit();
    }
    for (int kt = 0; kt < ktiles; ++kt) {
        cp_async_wait<kV2Stages - 2>();
        __syncthreads();
        if (kt + kV2Stages - 1 < ktiles) issue(kt + kV2Stages - 1);
        cp_async_commit();
        v2_ktile<TN>(As + (kt % kV2Stages) * kV2AStage, Bs + (kt % kV2Stages) * kV2BStage, tx, ty, acc);
    }
    cp_async_wait<0>();
    __syncthreads();
}

// Stores the tile's accumulators (rows ty + 16 i, column groups h * GS +
// 4 tx) with bounds checks.
template <int TN>
__device__ __forceinline__ void v2_store(float* __restrict__ C, int M, int N, int ldc, int m0, int n0,
                                         const float2 (&acc)[8][TN / 2], float beta) {
    using T = V2T<TN>;
    const int tid = threadIdx.x;
    const int tx = tid % T::TX, ty = tid / T::TX;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int gm = m0 + ty + 16 * i;
        if (gm >= M) continue;
#pragma unroll
        for (int h = 0; h < T::NG; ++h) {
            const int gn = n0 + h * T::GS + tx * 4;
            float* crow = C + (size_t)gm * ldc + gn;
            float v[4] = {acc[i][2 * h].x, acc[i][2 * h].y, acc[i][2 * h + 1].x, acc[i][2 * h + 1].y};
            if (gn + 4 <= N) {
                if (beta != 0.f) add_old_vec<4>(crow, beta, v);
                stg_vec<4>(crow, v);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (gn + j < N) crow[j] = beta != 0.f ? __fmaf_rn(beta, crow[j], v[j]) : v[j];
            }
        }
    }
}

template <int TN>
__global__ void __launch_bounds__(V2T<TN>::Threads, 1)
    sgemm_v2_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int M, int N,
                    int K, int lda, int ldb, int ldc, float beta) {
    using T = V2T<TN>;
    extern __shared__ __align__(16) float v2_smem[];
    const int m0 = blockIdx.y * kV2BM, n0 = blockIdx.x * kV2BN;
    float2 acc[8][T::NP];  // acc[row][column pair]
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < T::NP; ++j) acc[i][j] = make_float2(0.f, 0.f);
    v2_mainloop<TN>(A, B, M, N, lda, ldb, m0, n0, 0, K, v2_smem, acc);
    v2_store<TN>(C, M, N, ldc, m0, n0, acc, beta);
}

// ------------------------------------------------------------ stream-K
// When the 128 x 128 tiles do not fill whole waves of the GPU, one CTA per SM
// takes an equal share of the (tile, 16-wide K step) units, in order: its
// share starts with the tail of one tile's K range, continues with whole
// tiles and ends with the head of another. A tile split between CTAs is
// finished by the CTA holding its K = 0 head (the "owner", which reaches it
// last): the others each park their partial sums in a per-CTA slot of a
// global workspace (64 KiB, [v][thread] float4) and raise their flag; the
// owner waits for each flag (bounded), adds the partials in CTA order and
// stores C. Each CTA has at most one such parked partial (its first
// segment), and owners only wait on higher-numbered CTAs, so with every CTA
// resident (cooperative launch) the waits always end. Deterministic: the
// summation order depends only on M, N, K and the SM count. A flag holds
// the launch's epoch (so a flag left raised by a launch that timed out is
// not mistaken for a fresh one), and the owner clears each flag it consumed
// (so a replayed CUDA graph, whose epoch is frozen, also starts clean).
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

constexpr int kSkThreads = V2T<kV2TNStreamK>::Threads;
__global__ void __launch_bounds__(kSkThreads, 1)
    sgemm_sk_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int M, int N,
                    int K, int lda, int ldb, int ldc, float beta, float4* __restrict__ ws,
                    unsigned* __restrict__ flags, unsigned epoch) {
    constexpr int TN = kV2TNStreamK;
    using T = V2T<TN>;
    extern __shared__ __align__(16) float v2_smem[];
    __shared__ int s_ok;
    const int tid = threadIdx.x;
    const int nt = (N + kV2BN - 1) / kV2BN, mt = (M + kV2BM - 1) / kV2BM;
    const int iters = (K + kV2BK - 1) / kV2BK;  // K steps per tile
    const long long U = (long long)mt * nt * iters;
    const int G = (int)gridDim.x, c = (int)blockIdx.x;
    auto share_begin = [&](int q) { return U * q / G; };
    long long u = share_begin(c);
    const long long u_end = share_begin(c + 1);
    while (u < u_end) {
        const int t = (int)(u / iters);
        const long long tile_u0 = (long long)t * iters;
        const int kb = (int)(u - tile_u0);
        const int ke = (int)min((long long)iters, u_end - tile_u0);
        const int m0 = (t / nt) * kV2BM, n0 = (t % nt) * kV2BN;
        float2 acc[8][T::NP];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < T::NP; ++j) acc[i][j] = make_float2(0.f, 0.f);
        v2_mainloop<TN>(A, B, M, N, lda, ldb, m0, n0, kb * kV2BK, min(K, ke * kV2BK), v2_smem, acc);
        if (kb != 0) {
            // Not the owner: park the partial tile, then raise the flag.
            float4* dst = ws + (size_t)c * (T::Park * T::Threads);
#pragma unroll
            for (int v = 0; v < T::Park; ++v) {
                const int i = v / (T::NP / 2), j = (v % (T::NP / 2)) * 2;
                __stcg(dst + v * T::Threads + tid,
                       make_float4(acc[i][j].x, acc[i][j].y, acc[i][j + 1].x, acc[i][j + 1].y));
            }
            __syncthreads();
            if (tid == 0) {
                __threadfence();
                st_release_gpu(flags + c, epoch);
            }
        } else {
            if (ke < iters) {
                // Owner of a split tile: add the partials of the CTAs whose
                // shares start inside this tile, in CTA order.
                const long long tile_u1 = tile_u0 + iters;
                for (int q = c + 1; q < G; ++q) {
                    const long long qb = share_begin(q), qe = share_begin(q + 1);
                    if (qb >= tile_u1) break;
                    if (qb == qe) continue;  // empty share: nothing parked
                    if (tid == 0) {
                        bool ok = ld_acquire_gpu(flags + q) == epoch;
                        if (!ok) {
                            const uint64_t t0 = globaltimer_ns();
                            uint32_t spins = 0;
                            while (!(ok = ld_acquire_gpu(flags + q) == epoch)) {
                                if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) {
                                    record_error(GPLK_STATUS_DEVICE_TIMEOUT, 0x0B01);
                                    break;
                                }
                            }
                        }
                        if (ok) flags[q] = 0u;  // consumed; nothing else touches it in this launch
                        s_ok = ok;
                    }
                    __syncthreads();
                    if (s_ok) {
                        const float4* src = ws + (size_t)q * (T::Park * T::Threads);
#pragma unroll
                        for (int v = 0; v < T::Park; ++v) {
                            const int i = v / (T::NP / 2), j = (v % (T::NP / 2)) * 2;
                            const float4 p4 = __ldcg(src + v * T::Threads + tid);
                            acc[i][j] = __fadd2_rn(acc[i][j], make_float2(p4.x, p4.y));
                            acc[i][j + 1] = __fadd2_rn(acc[i][j + 1], make_float2(p4.z, p4.w));
                        }
                    }
                    __syncthreads();  // s_ok is rewritten for the next contributor
                    if (qe >= tile_u1) break;
                }
            }
            v2_store<TN>(C, M, N, ldc, m0, n0, acc, beta);
        }
        u = tile_u0 + ke;
    }
}

static int launch_v2(const float* A, const float* B, float* C, int M, int N, int K, int lda, int ldb, int ldc,
                     float beta, cudaStream_t stream) {
    constexpr int TN = kV2TNDense;
    const int smem = (int)(sizeof(float) * kV2Stages * (kV2AStage + kV2BStage));
    static thread_local uint64_t configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1ull << dev))) {
        if (cudaFuncSetAttribute(sgemm_v2_kernel<TN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return GPLK_STATUS_LAUNCH_FAIL;
        configured |= 1ull << dev;
    }
    const int nt = (N + kV2BN - 1) / kV2BN, mt = (M + kV2BM - 1) / kV2BM;
    sgemm_v2_kernel<TN><<<dim3(nt, mt), V2T<TN>::Threads, smem, stream>>>(A, B, C, M, N, K, lda, ldb, ldc, beta);
    return launch_status(cudaGetLastError());
}

// The stream-K workspace is the caller's: a flag per CTA (the first 256
// bytes hold up to 64 flags, more take further 256-byte blocks) followed by
// one parked partial tile per CTA (64 KiB). A flag holds the launch's epoch.
// The epochs live on the host, per (device, workspace address): the first
// launch that sees a workspace zeroes its flags on the stream (an
// asynchronous memset, no allocation); every launch then takes the next
// epoch, so a flag left raised by a launch that timed out never reads as
// fresh to a later one.
constexpr size_t kSkPartBytes = (size_t)V2T<kV2TNStreamK>::Park * kSkThreads * sizeof(float4);

static size_t sk_flag_bytes(int ctas) { return (((size_t)ctas * sizeof(unsigned)) + 255) & ~(size_t)255; }
static size_t sk_workspace_bytes(int ctas) { return sk_flag_bytes(ctas) + (size_t)ctas * kSkPartBytes; }

struct SkEpoch {
    int device;
    const void* ws;
    int ctas;
    unsigned epoch;
};
static std::mutex g_sk_mu;
static std::vector<SkEpoch> g_sk_epochs;

static int launch_sk(const float* A, const float* B, float* C, int M, int N, int K, int lda, int ldb, int ldc,
                     float beta, int sm_count, void* workspace, cudaStream_t stream) {
    const int smem = (int)(sizeof(float) * kV2Stages * (kV2AStage + kV2BStage));
    int dev = 0;
    cudaGetDevice(&dev);
    static thread_local uint64_t configured = 0;
    if (!(configured & (1ull << dev))) {
        if (cudaFuncSetAttribute(sgemm_sk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return GPLK_STATUS_LAUNCH_FAIL;
        configured |= 1ull << dev;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sgemm_sk_kernel, kSkThreads, (size_t)smem) !=
            cudaSuccess ||
        per_sm < 1)
        return GPLK_STATUS_UNSUPPORTED;
    const int G = sm_count;
    unsigned* flags = static_cast<unsigned*>(workspace);
    float4* ws = reinterpret_cast<float4*>(static_cast<uint8_t*>(workspace) + sk_flag_bytes(G));
    unsigned epoch = 0;
    {
        std::lock_guard<std::mutex> lock(g_sk_mu);
        SkEpoch* e = nullptr;
        for (SkEpoch& x : g_sk_epochs)
            if (x.device == dev && x.ws == workspace && x.ctas == G) e = &x;
        if (!e) {
            if (g_sk_epochs.size() >= 256) g_sk_epochs.clear();  // forgotten workspaces are zeroed again
            if (cudaMemsetAsync(flags, 0, sk_flag_bytes(G), stream) != cudaSuccess) return GPLK_STATUS_LAUNCH_FAIL;
            g_sk_epochs.push_back(SkEpoch{dev, workspace, G, 0u});
            e = &g_sk_epochs.back();
        }
        if (++e->epoch == 0u) e->epoch = 1u;
        epoch = e->epoch;
    }
    void* args[] = {&A, &B, &C, &M, &N, &K, &lda, &ldb, &ldc, &beta, &ws, &flags, &epoch};
    if (cudaLaunchCooperativeKernel((const void*)sgemm_sk_kernel, dim3((unsigned)G), dim3(kSkThreads), args,
                                    (size_t)smem, stream) != cudaSuccess)
        return GPLK_STATUS_LAUNCH_FAIL;
    return launch_status(cudaGetLastError());
}

template <int BM, int BN, int BK, int TM, int TN>
static int launch(const float* A, const float* B, float* C, int M, int N, int K, int lda, int ldb,
                  int ldc, float beta, bool vec, cudaStream_t stream) {
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    if (vec) {
        sgemm_kernel<BM, BN, BK, TM, TN, true><<<grid, Cfg<BM, BN, BK, TM, TN, true>::kThreads, 0, stream>>>(
            A, B, C, M, N, K, lda, ldb, ldc, beta);
    } else {
        sgemm_kernel<BM, BN, BK, TM, TN, false><<<grid, Cfg<BM, BN, BK, TM, TN, false>::kThreads, 0, stream>>>(
            A, B, C, M, N, K, lda, ldb, ldc, beta);
    }
    return launch_status(cudaGetLastError());
}

// Which kernel a problem takes (the 16-byte-aligned case decides the
// workspace size: only stream-K needs one).
enum class Plan { StreamK, V2, Tiles128, Split2, Tiles64 };

static Plan plan(int M, int N, int K, bool vec, int sm_count) {
    // 128 x 128 tiles. When they leave more than a tenth of the last wave's
    // SMs idle, stream-K spreads the K steps evenly over one CTA per SM;
    // tiny or shallow problems fall back to 64 x 64 tiles.
    const long tiles128 = (long)((M + 127) / 128) * ((N + 127) / 128);
    if (vec) {
        const long waves = (tiles128 + sm_count - 1) / sm_count;
        const bool ragged = tiles128 * 10 < waves * sm_count * 9;
        if (K >= 256 && 4 * tiles128 >= sm_count && ragged) return Plan::StreamK;
        if (tiles128 * 2 >= sm_count / 4) return Plan::V2;
    }
    if (tiles128 >= sm_count) return Plan::Tiles128;
    if (K >= 256 && 2 * tiles128 >= sm_count / 2) return Plan::Split2;
    return Plan::Tiles64;
}

}  // namespace sgemm
}  // namespace gplk

extern "C" size_t gplk_sgemm_workspace_bytes(int M, int N, int K) {
    using namespace gplk;
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    DeviceInfo d;
    if (current_device_info(&d) != GPLK_STATUS_OK) return 0;
    return sgemm::plan(M, N, K, true, d.sm_count) == sgemm::Plan::StreamK ? sgemm::sk_workspace_bytes(d.sm_count)
                                                                          : 0;
}

extern "C" int gplk_sgemm_f32(const float* A, const float* B, float* C, int M, int N, int K, int lda, int ldb,
                              int ldc, float beta, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    using namespace gplk;
    if (M < 0 || N < 0 || K < 0) return GPLK_STATUS_BAD_ARG;
    if (M == 0 || N == 0) return GPLK_STATUS_OK;
    if (!C || (K > 0 && (!A || !B))) return GPLK_STATUS_BAD_ARG;  // K == 0: A, B unread
    if ((K > 0 && (lda < K || ldb < N)) || ldc < N) return GPLK_STATUS_BAD_ARG;
    if (workspace && !aligned16(workspace)) return GPLK_STATUS_BAD_ARG;
    DeviceInfo d;
    int st = current_device_info(&d);
    if (st != GPLK_STATUS_OK) return st;
    const bool vec = aligned16(A) && aligned16(B) && aligned16(C) && (lda % 4 == 0) && (ldb % 4 == 0) &&
                     (ldc % 4 == 0) && (K % 4 == 0) && (N % 4 == 0);
    switch (sgemm::plan(M, N, K, vec, d.sm_count)) {
        case sgemm::Plan::StreamK:
            if (workspace && workspace_bytes >= sgemm::sk_workspace_bytes(d.sm_count)) {
                st = sgemm::launch_sk(A, B, C, M, N, K, lda, ldb, ldc, beta, d.sm_count, workspace, stream);
                if (st != GPLK_STATUS_UNSUPPORTED) return st;
            }
            // No (or too small a) workspace: the whole-tile kernel instead.
            return sgemm::launch_v2(A, B, C, M, N, K, lda, ldb, ldc, beta, stream);
        case sgemm::Plan::V2:
            return sgemm::launch_v2(A, B, C, M, N, K, lda, ldb, ldc, beta, stream);
        case sgemm::Plan::Tiles128:
            return sgemm::launch<128, 128, 16, 8, 8>(A, B, C, M, N, K, lda, ldb, ldc, beta, vec, stream);
        case sgemm::Plan::Split2:
            return sgemm::launch_split2(A, B, C, M, N, K, lda, ldb, ldc, beta, vec, stream);
        default:
            return sgemm::launch<64, 64, 16, 4, 4>(A, B, C, M, N, K, lda, ldb, ldc, beta, vec, stream);
    }
}
