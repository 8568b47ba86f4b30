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
                        int N, int K, int lda, int ldb, int ldc) {
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
                const float* val = &acc[h * TM2 + i][g * TN2];
                if (VEC && gn + TN2 <= N) {
                    stg_vec<TN2>(crow, val);
                } else {
#pragma unroll
                    for (int j = 0; j < TN2; ++j)
                        if (gn + j < N) crow[j] = val[j];
                }
            }
        }
    }
}

static int launch_split2(const float* A, const float* B, float* C, int M, int N, int K, int lda, int ldb, int ldc,
                         bool vec, cudaStream_t stream) {
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
        sgemm_split2_kernel<true><<<grid, kSplitThreads, smem, stream>>>(A, B, C, M, N, K, lda, ldb, ldc);
    else
        sgemm_split2_kernel<false><<<grid, kSplitThreads, smem, stream>>>(A, B, C, M, N, K, lda, ldb, ldc);
    return launch_status(cudaGetLastError());
}

// ------------------------------------------------------------ cp.async + FFMA2 main loop
// 128 x 128 tiles, 256 threads, 8 x 8 outputs per thread (rows ty*4+i and
// 64+ty*4+i, columns tx*4+j and 64+tx*4+j), BK = 16, a 3-stage ring filled
// by cp.async straight from global memory (no register staging). A stays
// K-major in shared memory (one 128-bit load = four k of one row), B stays
// N-major. The FFMAs issue as Blackwell's paired FP32 FMA (__ffma2_rn: two
// independent, individually rounded fmaf per instruction) on column pairs,
// halving the FMA issue slots. Each output is still one FMA chain over k in
// order. SPLIT: 2-CTA cluster split-K with a distributed-shared-memory sum.
constexpr int kV2BM = 128, kV2BN = 128, kV2BK = 16, kV2Stages = 3, kV2Threads = 256;
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

template <bool SPLIT>
__global__ void __launch_bounds__(kV2Threads, 1) sgemm_v2_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                                  float* __restrict__ C, int M, int N, int K, int lda,
                                                                  int ldb, int ldc) {
    extern __shared__ __align__(16) float v2_smem[];
    float* As = v2_smem;                          // [stage][128][kV2APitch]
    float* Bs = v2_smem + kV2Stages * kV2AStage;  // [stage][16][128]
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const int m0 = blockIdx.y * kV2BM;
    const uint32_t rank = SPLIT ? cluster_ctarank() : 0u;
    const int n0 = (SPLIT ? (blockIdx.x >> 1) : blockIdx.x) * kV2BN;
    int k_begin = 0, k_end = K;
    if (SPLIT) {
        const int k_half = ((K + 2 * kV2BK - 1) / (2 * kV2BK)) * kV2BK;
        k_begin = rank == 0 ? 0 : k_half;
        k_end = rank == 0 ? min(K, k_half) : K;
    }
    const int ktiles = k_end > k_begin ? (k_end - k_begin + kV2BK - 1) / kV2BK : 0;

    // Each thread copies 2 A chunks (row r, k-quad q) and 2 B chunks.
    auto issue = [&](int kt) {
        const int st = kt % kV2Stages;
        const int k0 = k_begin + kt * kV2BK;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + i * kV2Threads;  // 0..511
            const int r = idx >> 2, q = idx & 3;
            const int gm = m0 + r, gk = k0 + q * 4;
            const bool ok = gm < M && gk < k_end;
            cp_async16(As + st * kV2AStage + r * kV2APitch + q * 4, ok ? A + (size_t)gm * lda + gk : A, ok);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int idx = tid + i * kV2Threads;
            const int r = idx >> 5, c4 = idx & 31;
            const int gk = k0 + r, gn = n0 + c4 * 4;
            const bool ok = gk < k_end && gn < N;
            cp_async16(Bs + st * kV2BStage + r * kV2BN + c4 * 4, ok ? B + (size_t)gk * ldb + gn : B, ok);
        }
    };

    float2 acc[8][4];  // acc[row][column pair]
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.f, 0.f);

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
        const float* as = As + (kt % kV2Stages) * kV2AStage;
        const float* bs = Bs + (kt % kV2Stages) * kV2BStage;
#pragma unroll
        for (int kq = 0; kq < kV2BK; kq += 4) {
            float4 af[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int row = (i >> 2) * 64 + ty * 4 + (i & 3);
                af[i] = *reinterpret_cast<const float4*>(as + row * kV2APitch + kq);
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const float4 b0 = *reinterpret_cast<const float4*>(bs + (kq + kk) * kV2BN + tx * 4);
                const float4 b1 = *reinterpret_cast<const float4*>(bs + (kq + kk) * kV2BN + 64 + tx * 4);
                const float2 bp[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                                      make_float2(b1.z, b1.w)};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float av = kk == 0 ? af[i].x : kk == 1 ? af[i].y : kk == 2 ? af[i].z : af[i].w;
                    const float2 a2 = make_float2(av, av);
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = __ffma2_rn(a2, bp[j], acc[i][j]);
                }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    if (SPLIT) {
        // CTA 1 hands its partial tile to CTA 0 through distributed shared
        // memory ([v][thread] float4 layout, contiguous per warp).
        // The receive buffer has its own region after the operand ring, so
        // CTA 1 may write it while CTA 0 still reads its last stage.
        float4* recv = reinterpret_cast<float4*>(v2_smem + kV2Stages * (kV2AStage + kV2BStage));
        if (rank == 1) {
            const uint32_t dst0 = mapa_shared(smem_u32(recv), 0);
#pragma unroll
            for (int v = 0; v < 16; ++v) {
                const int i = v >> 1, j = (v & 1) * 2;
                const uint32_t addr = dst0 + (uint32_t)((v * kV2Threads + tid) * 16);
                asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(acc[i][j].x),
                             "f"(acc[i][j].y), "f"(acc[i][j + 1].x), "f"(acc[i][j + 1].y)
                             : "memory");
            }
        }
        cluster_sync();
        if (rank == 1) return;
#pragma unroll
        for (int v = 0; v < 16; ++v) {
            const int i = v >> 1, j = (v & 1) * 2;
            const float4 q = recv[v * kV2Threads + tid];
            acc[i][j] = __fadd2_rn(acc[i][j], make_float2(q.x, q.y));
            acc[i][j + 1] = __fadd2_rn(acc[i][j + 1], make_float2(q.z, q.w));
        }
    }

#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int gm = m0 + (i >> 2) * 64 + ty * 4 + (i & 3);
        if (gm >= M) continue;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            const int gn = n0 + g * 64 + tx * 4;
            float* crow = C + (size_t)gm * ldc + gn;
            const float2 p0 = acc[i][2 * g], p1 = acc[i][2 * g + 1];
            if (gn + 4 <= N) {
                *reinterpret_cast<float4*>(crow) = make_float4(p0.x, p0.y, p1.x, p1.y);
            } else {
                const float v4[4] = {p0.x, p0.y, p1.x, p1.y};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (gn + j < N) crow[j] = v4[j];
            }
        }
    }
}

template <bool SPLIT>
static int launch_v2(const float* A, const float* B, float* C, int M, int N, int K, int lda, int ldb, int ldc,
                     cudaStream_t stream) {
    int smem = (int)(sizeof(float) * kV2Stages * (kV2AStage + kV2BStage));
    if (SPLIT) smem += (int)(16 * kV2Threads * sizeof(float4));
    static thread_local uint64_t configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1ull << dev))) {
        if (cudaFuncSetAttribute(sgemm_v2_kernel<SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return GPLK_STATUS_LAUNCH_FAIL;
        configured |= 1ull << dev;
    }
    const int nt = (N + kV2BN - 1) / kV2BN, mt = (M + kV2BM - 1) / kV2BM;
    if (!SPLIT) {
        sgemm_v2_kernel<false><<<dim3(nt, mt), kV2Threads, smem, stream>>>(A, B, C, M, N, K, lda, ldb, ldc);
    } else {  // clusters of two along x, set at launch
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * nt, mt, 1);
        cfg.blockDim = dim3(kV2Threads, 1, 1);
        cfg.dynamicSmemBytes = (size_t)smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&cfg, sgemm_v2_kernel<true>, A, B, C, M, N, K, lda, ldb, ldc) != cudaSuccess)
            return GPLK_STATUS_LAUNCH_FAIL;
    }
    return launch_status(cudaGetLastError());
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
    // 128 x 128 tiles (8 x 8 per thread). When they cannot fill the GPU, a
    // 2-CTA cluster splits K per tile (each tile then occupies two SMs); tiny
    // or shallow problems fall back to 64 x 64 tiles.
    const long tiles128 = (long)((M + 127) / 128) * ((N + 127) / 128);
    if (vec) {  // 16-byte aligned rows: the cp.async + FFMA2 kernel
        if (tiles128 >= d.sm_count) return sgemm::launch_v2<false>(A, B, C, M, N, K, lda, ldb, ldc, stream);
        if (K >= 256 && 2 * tiles128 >= d.sm_count / 2)
            return sgemm::launch_v2<true>(A, B, C, M, N, K, lda, ldb, ldc, stream);
        if (tiles128 * 2 >= d.sm_count / 4)
            return sgemm::launch_v2<false>(A, B, C, M, N, K, lda, ldb, ldc, stream);
    }
    if (tiles128 >= d.sm_count)
        return sgemm::launch<128, 128, 16, 8, 8>(A, B, C, M, N, K, lda, ldb, ldc, vec, stream);
    if (K >= 256 && 2 * tiles128 >= d.sm_count / 2)
        return sgemm::launch_split2(A, B, C, M, N, K, lda, ldb, ldc, vec, stream);
    return sgemm::launch<64, 64, 16, 4, 4>(A, B, C, M, N, K, lda, ldb, ldc, vec, stream);
}
