// gplk_gemm_pair.cu - tcgen05 GEMMs on CTA pairs, one kernel template for
// every dense precision of the GEMM ladder:
//
//   FP8   E4M3 x E4M3 -> FP32 accumulate -> scaled BF16  kind::f8f6f4, K = 32 / MMA
//         cuBLASLt's TN layout (runner/src/gemm_lt.cu:98-132): A and B
//         K-major, per-tensor FP32 scales
//   BF16  BF16 x BF16 -> FP32 accumulate -> BF16   kind::f16,  K = 16 / MMA
//   FP16  FP16 x FP16 -> FP32 accumulate -> FP16   kind::f16,  K = 16 / MMA
//   TF32  FP32 x FP32 (TF32 products) -> FP32       kind::tf32, K =  8 / MMA
//   INT8  S8 x S8 -> S32 accumulate -> S32          kind::i8,   K = 32 / MMA
//         the last four in the layout of the reference's cublasGemmEx rung
//         (runner/src/workload_gemm.c:44-79 maps them, :155-163 calls them):
//         all matrices column-major, C = A * B with no transposes, alpha 1,
//         beta 0 -- or beta 1 (C = A * B + C, the powervirus tensor stream's
//         call, runner/src/workload_powervirus.cu:363-380): the epilogue
//         then reads the old C element, adds it to the FP32 / S32 sum and
//         rounds once. Column-major A (M x K) has M contiguous, so the MMA
//         reads it MN-major; column-major B (K x N) is K-major. The reference
//         computes FP16 with CUBLAS_COMPUTE_16F; here FP16 accumulates in
//         FP32 (at least as accurate) and rounds once to FP16.
// D is always M x N column-major.
//
// A persistent grid of 2-CTA clusters walks 256 x BN output tiles (BN = 256;
// 128 for problems too small to fill the SMs with 256-wide tiles, see
// tile_plan; a short last wave of 256-wide tiles runs as 256 x 128 halves,
// see item_tile) in a grouped order (raster groups along M; odd groups walk N
// backwards). It is
// launched with programmatic stream serialisation, so its set-up overlaps
// the previous GEMM on the stream. Per cluster, one tcgen05.mma.cta_group::2 (M = 256,
// N = 256) per 32 bytes of K; each CTA TMA-loads its own 128 rows of the A
// tile and its own 128 rows (N) of the B tile with the 128-byte swizzle, no
// cluster multicast. A pipeline stage holds two 128-byte slabs of K (64 KiB
// per CTA, 8 MMAs), three stages deep: the leader's MMA thread waits on one
// barrier and releases the stage in both CTAs with one commit per CTA every
// 8 MMAs, not every 4. (On B200 the per-stage wait-and-commit sequence costs
// tensor-pipe time: 4-MMA stages measured 3602 TFLOP/s for FP8 8192^3, 8-MMA
// stages 4092.) The FP32/S32 accumulator is double-buffered in TMEM
// (2 x 256 columns) so the epilogue of one tile overlaps the main loop of
// the next. The epilogue converts, stages 8 KiB column chunks in shared
// memory and writes them with TMA stores. Every wait is bounded (2 s); on
// timeout the kernel records GPLK_STATUS_DEVICE_TIMEOUT with the site,
// drains and returns.
#include <cstring>

#include "gplk_ptx.cuh"

namespace gplk {
namespace pair {

enum class Kind { F8F6F4, F16, TF32, I8 };
enum class Out { BF16, F16, F32, S32 };

constexpr int kThreads = 192;
constexpr int kSlab = 128 * 128;          // one CTA's 128 rows x 128 bytes of K
constexpr int kSlabs = 2;                 // K slabs per stage (8 MMAs)
constexpr int kOperandBytes = kSlabs * kSlab;    // A part of a stage: 32 KiB

// Pair-tile geometry for tile width BN (the pair computes 256 x BN; each CTA
// holds 128 rows of A and BN / 2 rows of B per K slab). Narrower tiles have
// smaller stages, so their rings are deeper in the same shared memory.
template <int BN>
struct Geom {
    static_assert(BN == 256 || BN == 128, "pair tile width");
    static constexpr int kBRows = BN / 2;
    static constexpr int kBSlab = kBRows * 128;
    static constexpr int kBOperand = kSlabs * kBSlab;
    static constexpr int kStageBytes = kOperandBytes + kBOperand;  // 64 / 48 KiB per CTA
    static constexpr int kStages = BN == 256 ? 3 : 4;
    static constexpr int kBBox = 64;  // rows of B per TMA box (two per slab for BN = 256)
    static constexpr uint32_t kTmemCols = 2u * (uint32_t)BN;  // double-buffered accumulator
};
constexpr int kMaxGroupM = 16;            // raster group along M (pair tiles), bounds
constexpr int kMinGroupM = 8;
#ifndef GPLK_PAIR_PANEL_BUDGET
#define GPLK_PAIR_PANEL_BUDGET (32u << 20)
#endif
// Bytes of A row panels a raster group may keep live in L2: a group of g
// pair-tiles along M shares g panels of 256 rows x K of A while it walks N.
constexpr size_t kPanelBudget = GPLK_PAIR_PANEL_BUDGET;
constexpr int kOutChunkBytes = 8192;      // epilogue staging: 8 KiB column chunks

// Operand kind, A/B element format code in the instruction descriptor,
// output type, A's major-ness (B is always K-major) and whether D is scaled
// by per-tensor scales.
template <Kind KIND, uint32_t FMT, Out OUT, bool A_KMAJOR = false, bool SCALED = false>
struct Cfg {
    static constexpr Kind kKind = KIND;
    static constexpr Out kOut = OUT;
    static constexpr bool kAKMajor = A_KMAJOR;
    static constexpr bool kScaled = SCALED;
    static constexpr int kInBytes = KIND == Kind::F16 ? 2 : KIND == Kind::TF32 ? 4 : 1;
    static constexpr int kOutBytes = (OUT == Out::BF16 || OUT == Out::F16) ? 2 : 4;
    static constexpr int kRowElems = 128 / kInBytes;  // elements per 128-byte run = K per stage
    // MN-major A: the CTA's 128 rows of M are 128 / kRowElems runs of
    // kRowElems elements; each run is one TMA box of kRowElems (M) x
    // kRowElems (K) and one swizzle-atom column of the MMA's A operand.
    static constexpr int kABoxes = A_KMAJOR ? 1 : 128 / kRowElems;
    static constexpr uint32_t kABoxBytes = (uint32_t)kSlab / (uint32_t)kABoxes;
    // One MMA consumes 32 bytes of K: 32 / kInBytes K rows of 128 bytes in
    // the MN-major A tile, 32 bytes along each 128-byte row of B.
    static constexpr uint32_t kAStep = (32u / (uint32_t)kInBytes) * 128u;
    // Swizzle of the MN-major A tile. 16- and 8-bit operands use the 128-byte
    // swizzle of 16-byte units (8-row, 1024-byte atoms). An MN-major TF32
    // operand must use the 128-byte swizzle of 32-byte units instead (the
    // MMA's SWIZZLE_128B_BASE32B layout, 4-row 512-byte atoms), which TMA
    // writes with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.
    static constexpr bool kA32BAtoms = KIND == Kind::TF32;
    static constexpr uint32_t kADescLayout = kA32BAtoms ? 1u : 2u;
    static constexpr uint32_t kASbo = kA32BAtoms ? 512u : 1024u;
    static constexpr int kChunkCols = kOutChunkBytes / (128 * kOutBytes);  // 32 or 16
    // Instruction descriptor (M = 256, N = n, B K-major).
    __host__ __device__ static constexpr uint32_t idesc(uint32_t n) {
        return ((KIND == Kind::I8 ? 2u : 1u) << 4)  // D: S32 or F32
               | (FMT << 7) | (FMT << 10)           // A, B formats
               | ((A_KMAJOR ? 0u : 1u) << 15)       // A major-ness
               | ((n >> 3) << 17) | ((256u >> 4) << 24);
    }
};

using CfgFP8 = Cfg<Kind::F8F6F4, 0u, Out::BF16, true, true>;  // F8F6F4 format 0 = E4M3
using CfgBF16 = Cfg<Kind::F16, 1u, Out::BF16>;  // F16F32 format 1 = BF16
using CfgF16 = Cfg<Kind::F16, 0u, Out::F16>;    // F16F32 format 0 = F16
using CfgTF32 = Cfg<Kind::TF32, 2u, Out::F32>;  // F16F32 format 2 = TF32
using CfgI8 = Cfg<Kind::I8, 1u, Out::S32>;      // S8 format 1 = signed

template <Kind KIND>
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    if constexpr (KIND == Kind::F8F6F4) {
        mma_pair_f8f6f4(d_tmem, a_desc, b_desc, idesc, accumulate);
    } else if constexpr (KIND == Kind::F16) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else if constexpr (KIND == Kind::TF32) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// MN-major A tile: runs of 128 bytes along M, one K row per run, swizzle
// atoms of `sbo` bytes along K (layout 2: 8 rows, 16-byte units; layout 1:
// 4 rows, 32-byte units); the next run of M starts `lbo` bytes on.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t start, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return smem_desc(start, lbo, sbo, layout);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// acc + old for beta = 1, in the accumulator's type: FP32 add (the old
// BF16 / FP16 value widened exactly) or wrapping S32 add. The sum is then
// rounded once to the output type by the epilogue, as cuBLAS computes
// alpha * acc + beta * C with alpha = beta = 1.
template <Out OUT>
__device__ __forceinline__ uint32_t add_old(uint32_t acc_bits, uint32_t old) {
    if constexpr (OUT == Out::S32) {
        return (uint32_t)((int32_t)acc_bits + (int32_t)old);
    } else if constexpr (OUT == Out::F32) {
        return __float_as_uint(__fadd_rn(__uint_as_float(acc_bits), __uint_as_float(old)));
    } else if constexpr (OUT == Out::BF16) {
        return __float_as_uint(__fadd_rn(__uint_as_float(acc_bits), __uint_as_float(old << 16)));
    } else {
        float h;
        asm("cvt.f32.f16 %0, %1;" : "=f"(h) : "h"((unsigned short)old));
        return __float_as_uint(__fadd_rn(__uint_as_float(acc_bits), h));
    }
}

struct Params {
    void* D;
    const float* scale_a;  // FP8: per-tensor scales (device pointers)
    const float* scale_b;
    int M, N, K;  // K in elements
    int m_tiles, n_tiles, k_stages;
    int group_m;    // raster group along M (pair tiles)
    int tma_store;  // stage the epilogue through shared memory and TMA-store it
    int accumulate; // beta = 1: D = A * B + D (D read before it is written)
    // Work items: items below full_items are whole pair tiles (item = tile);
    // the rest split the last wave's 256 x 256 tiles into 256 x 128 halves.
    int full_items, num_items;
    int frag_store;  // 2-byte D, TMA stores, beta = 0: staged by stmatrix into swizzled 64-row boxes
};

// Work item -> pair tile and column half (-1: the whole 256 x BN tile).
__device__ __forceinline__ int item_tile(const Params& p, int item, int& half) {
    if (item < p.full_items) {
        half = -1;
        return item;
    }
    const int u = item - p.full_items;
    half = u & 1;
    return p.full_items + (u >> 1);
}

template <int BN>
struct __align__(1024) Smem {
    uint8_t stage[Geom<BN>::kStages][Geom<BN>::kStageBytes];
    uint8_t out_stage[2][kOutChunkBytes];
    uint64_t full[Geom<BN>::kStages];
    uint64_t empty[Geom<BN>::kStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
    int epi_fail;
};

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int group_m, int& mt, int& nt) {
    const int per_group = group_m * n_tiles;
    const int group = t / per_group;
    const int first_m = group * group_m;
    const int gsize = min(m_tiles - first_m, group_m);
    const int r = t % per_group;
    mt = first_m + r % gsize;
    nt = r / gsize;
    // Odd groups walk N backwards, so the first wave of a group reuses the B
    // column panels the last wave of the previous group left in L2.
    if (group & 1) nt = n_tiles - 1 - nt;
}

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 32) {
        tmem_ld_32x32b_x32(taddr, r);
    } else {
        static_assert(N == 16, "16 or 32 columns per load");
        tmem_ld_32x32b_x16(taddr, r);
    }
}

template <class C, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmD, const Params p) {
    using G = Geom<BN>;
    constexpr int S = G::kStages;
    constexpr int kChunks = BN / C::kChunkCols;
    static_assert(kChunks % 2 == 0, "the epilogue handles chunks in pairs");
    extern __shared__ uint8_t smem_raw[];
    Smem<BN>& sm =
        *reinterpret_cast<Smem<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t warp = warp_id_uniform();
    const uint32_t lane = lane_id();
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster = (int)(blockIdx.x >> 1);
    const int nclusters = (int)(gridDim.x >> 1);

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.acc_full[i], 1);
            mbar_init(&sm.acc_empty[i], 8);  // four epilogue warps in each CTA of the pair
        }
        mbar_init(&sm.drain, 1);
        sm.abort = 0;
        sm.epi_fail = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (p.tma_store) tma_prefetch_desc(&tmD);
    }
    if (warp == 1) {
        tmem_alloc_pair(&sm.tmem_base, G::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    // Launched with programmatic stream serialisation: the set-up above may
    // overlap the previous kernel's tail; nothing below touches global
    // memory before that kernel has completed. The next GEMM on the stream
    // may then be launched into SMs as they free up.
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        // TMA producer (one thread per CTA); both CTAs' bytes complete on the
        // leader's `full` barrier.
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, issued_parity = 0;
            bool ok = true;
            for (int it = cluster; it < p.num_items && ok; it += nclusters) {
                int half;
                const int t = item_tile(p, it, half);
                int mt, nt;
                tile_coords(t, p.m_tiles, p.n_tiles, p.group_m, mt, nt);
                const int m_base = mt * 256 + (int)rank * 128;
                // This CTA's B rows: kBRows of the tile, or, for a half item,
                // its half's kBRows / 2 (the pair's N = 128 split over both
                // CTAs), loaded into the first half of each slab's B region.
                const int b_row = half < 0 ? nt * BN + (int)rank * G::kBRows
                                           : nt * BN + 128 * half + (int)rank * (G::kBRows / 2);
                const uint32_t stage_tx =
                    half < 0 ? 2u * (uint32_t)G::kStageBytes : 2u * (uint32_t)(kOperandBytes + G::kBOperand / 2);
                for (int kb = 0; kb < p.k_stages; ++kb) {
                    if (!mbar_wait_cluster(&sm.empty[stage], phase ^ 1u, &sm.abort, 0x0501)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = sm.stage[stage];
                    const uint32_t full_leader = mapa_shared(smem_u32(&sm.full[stage]), 0);
                    if (leader) mbar_arrive_expect_tx(&sm.full[stage], stage_tx);
#pragma unroll
                    for (int sl = 0; sl < kSlabs; ++sl) {
                        const int kk = kb * kSlabs + sl;  // 128-byte slab of K
                        uint8_t* a_dst = st + sl * kSlab;
                        if constexpr (C::kAKMajor) {
                            tma_load_2d_pair(a_dst, &tmA, full_leader, kk * 128, m_base);
                        } else {
#pragma unroll
                            for (int b = 0; b < C::kABoxes; ++b)
                                tma_load_2d_pair(a_dst + b * C::kABoxBytes, &tmA, full_leader,
                                                 (m_base + b * C::kRowElems) * C::kInBytes, kk * C::kRowElems);
                        }
                        // B in boxes of kBBox = 64 rows: one per slab for a
                        // 128-wide tile or a half item, two for a 256-wide tile.
                        uint8_t* b_dst = st + kOperandBytes + sl * G::kBSlab;
                        tma_load_2d_pair(b_dst, &tmB, full_leader, kk * 128, b_row);
                        if (half < 0 && G::kBBox < G::kBRows)
                            tma_load_2d_pair(b_dst + G::kBBox * 128, &tmB, full_leader, kk * 128, b_row + G::kBBox);
                    }
                    issued_mask |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (leader && (!ok || sm.abort)) {
                int dummy = 0;
                for (int s2 = 0; s2 < S; ++s2)
                    if (issued_mask & (1u << s2))
                        mbar_wait_cluster(&sm.full[s2], (issued_parity >> s2) & 1u, &dummy, 0x0502, 100000000ull);
            }
        }
    } else if (warp == 1) {
        // MMA issuer: the leader's one thread.
        if (leader && lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int it = cluster; it < p.num_items && ok; it += nclusters) {
                int half;
                (void)item_tile(p, it, half);
                const uint32_t idesc = C::idesc(half < 0 ? (uint32_t)BN : 128u);
                if (!mbar_wait_cluster(&sm.acc_empty[acc], acc_phase ^ 1u, &sm.abort, 0x0511)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)acc * (uint32_t)BN;
                for (int kb = 0; kb < p.k_stages; ++kb) {
                    if (!mbar_wait_cluster(&sm.full[stage], phase, &sm.abort, 0x0512)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sm.stage[stage]);
                    const uint32_t b_addr = a_addr + kOperandBytes;
#pragma unroll
                    for (int j = 0; j < 4 * kSlabs; ++j) {
                        const uint32_t slab = (uint32_t)(j >> 2) * kSlab, jj = (uint32_t)(j & 3);
                        const uint32_t bslab = (uint32_t)(j >> 2) * (uint32_t)G::kBSlab;
                        const uint64_t a_desc =
                            C::kAKMajor ? desc_kmajor_sw128(a_addr + slab + 32u * jj)
                                        : desc_mnmajor(a_addr + slab + C::kAStep * jj, C::kABoxBytes, C::kASbo,
                                                       C::kADescLayout);
                        mma_pair<C::kKind>(d_tmem, a_desc, desc_kmajor_sw128(b_addr + bslab + 32u * jj),
                                           idesc, (kb | j) != 0);
                    }
                    const uint32_t e = smem_u32(&sm.empty[stage]);
                    tc_commit_pair(mapa_shared(e, 0));
                    tc_commit_pair(mapa_shared(e, 1));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                const uint32_t f = smem_u32(&sm.acc_full[acc]);
                tc_commit_pair(mapa_shared(f, 0));
                tc_commit_pair(mapa_shared(f, 1));
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            tc_commit_pair(mapa_shared(smem_u32(&sm.drain), 0));
            int dummy = 0;
            mbar_wait_cluster(&sm.drain, 0, &dummy, 0x0513, 100000000ull);
        }
    } else {
        // Epilogue: warps 2..5 read TMEM lanes 32*(warp%4).. (= rows of this
        // CTA's 128-row half), convert, and stage each column chunk as
        // [column][row] in shared memory for one TMA store.
        constexpr int CC = C::kChunkCols;
        const float scale = C::kScaled ? __ldg(p.scale_a) * __ldg(p.scale_b) : 1.0f;
        const uint32_t quarter = warp & 3u;
        const int row_in_half = (int)(quarter * 32 + lane);
        const bool issuer = warp == 2 && lane == 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t chunk_seq = 0;
        for (int it = cluster; it < p.num_items; it += nclusters) {
            int half;
            const int t = item_tile(p, it, half);
            int mt, nt;
            tile_coords(t, p.m_tiles, p.n_tiles, p.group_m, mt, nt);
            const int nch = half < 0 ? kChunks : kChunks / 2;  // chunks of this item (even)
            if (!mbar_wait_sleepy(&sm.acc_full[acc], acc_phase, &sm.abort, 0x0521, true)) sm.epi_fail = 1;
            named_sync(1, 128);
            if (*(volatile int*)&sm.epi_fail) break;
            tc_fence_after();
            const int m0 = mt * 256 + (int)rank * 128;
            const int m = m0 + row_in_half;
            const int n_base = nt * BN + (half > 0 ? 128 : 0);
            const uint32_t t_addr = tmem + ((quarter * 32u) << 16) + (uint32_t)acc * (uint32_t)BN;
            const uint32_t acc_empty_leader = mapa_shared(smem_u32(&sm.acc_empty[acc]), 0);
            bool staged = false;
            if constexpr (C::kOutBytes == 2) {
                if (p.frag_store) {
                    // 2-byte D with TMA stores, beta = 0. Per 32-column chunk
                    // each warp loads its 32 rows as two 16-lane
                    // tcgen05.ld.16x256b.x4 (mma-fragment registers: thread t
                    // holds rows t/4 and t/4 + 8 at columns 2(t%4), +1 of every
                    // 8-column group), converts, and stages them with
                    // stmatrix .trans in the 128-byte-swizzled layout of two
                    // 64-row x 32-column TMA boxes: 16 conflict-free wavefronts
                    // per warp and chunk instead of 32.
                    const uint32_t lanes0 = t_addr;
                    const uint32_t lanes1 = t_addr + (16u << 16);
                    const int r0 = (int)quarter * 32 + 8 * (int)(lane >> 3);
                    const uint32_t jr = lane & 7u;
                    const uint32_t box_off = (uint32_t)(r0 >> 6) * 4096u;
                    const uint32_t chk = (uint32_t)((r0 & 63) >> 3);
                    auto fchunk = [&](int c, uint32_t (&x)[2][16]) {
                        tmem_ld_16x256b_x4(lanes0 + 32u * (uint32_t)c, x[0]);
                        tmem_ld_16x256b_x4(lanes1 + 32u * (uint32_t)c, x[1]);
                        tmem_ld_wait();
                        if (c + 1 == nch) {  // the whole accumulator is in registers: release it
                            tc_fence_before();
                            __syncwarp();
                            if (lane == 0) mbar_arrive_cluster(acc_empty_leader);
                        }
                        uint8_t* stg = sm.out_stage[chunk_seq & 1u];
                        if (issuer) bulk_wait_read<1>();  // the store that last used this buffer has read it
                        named_sync(1, 128);
                        const uint32_t sbase = smem_u32(stg) + box_off;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint32_t cc = (uint32_t)(8 * k) + jr;  // D column within the chunk
                            const uint32_t addr = sbase + cc * 128u + ((chk ^ (cc & 7u)) << 4);
                            auto pk = [&](int h, int i) {
                                const float lo = __uint_as_float(x[h][i]) * scale;
                                const float hi = __uint_as_float(x[h][i + 1]) * scale;
                                return C::kOut == Out::BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
                            };
                            stmatrix_x4_trans(addr, pk(0, 4 * k), pk(0, 4 * k + 2), pk(1, 4 * k), pk(1, 4 * k + 2));
                        }
                        fence_proxy_async_smem();
                        named_sync(1, 128);
                        if (issuer && n_base + CC * c < p.N) {
                            if (m0 < p.M) tma_store_2d(&tmD, stg, m0, n_base + CC * c);
                            if (m0 + 64 < p.M) tma_store_2d(&tmD, stg + 4096, m0 + 64, n_base + CC * c);
                            bulk_commit();
                        }
                        ++chunk_seq;
                    };
                    uint32_t xa[2][16];
#pragma unroll 1
                    for (int c = 0; c < nch; ++c) fchunk(c, xa);
                    staged = true;
                }
            }
            if (!staged) {
            // One chunk of CC columns: chunk c's accumulator values are in
            // `r` (loaded and waited for); the TMEM load of chunk c + 1 into
            // `nx` is issued before chunk c is converted and stored, so its
            // latency hides behind that work.
            auto chunk = [&](int c, uint32_t (&r)[CC], uint32_t (&nx)[CC]) {
                // beta = 1: this thread's row of the chunk's CC columns of the
                // old D (a warp reads 32 consecutive rows of one column: 64 or
                // 128 contiguous bytes).
                uint32_t old[CC];
                if (p.accumulate) {
                    const bool row_ok = m < p.M;
#pragma unroll
                    for (int j = 0; j < CC; ++j) {
                        const int n = n_base + CC * c + j;
                        old[j] = 0u;
                        if (row_ok && n < p.N) {
                            const size_t off = (size_t)n * (size_t)p.M + (size_t)m;
                            if constexpr (C::kOutBytes == 2)
                                old[j] = (uint32_t)__ldcs(static_cast<const uint16_t*>(p.D) + off);
                            else
                                old[j] = __ldcs(static_cast<const uint32_t*>(p.D) + off);
                        }
                    }
                }
                if (c + 1 < nch) {
                    tmem_ld_cols<CC>(t_addr + (uint32_t)(CC * (c + 1)), nx);
                } else {  // the whole accumulator is in registers: release it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(acc_empty_leader);
                }
                if (p.accumulate) {
#pragma unroll
                    for (int j = 0; j < CC; ++j) r[j] = add_old<C::kOut>(r[j], old[j]);
                }
                if (p.tma_store) {
                    uint8_t* stg = sm.out_stage[chunk_seq & 1u];
                    if (issuer) bulk_wait_read<1>();  // the store that last used this buffer has read it
                    named_sync(1, 128);
                    if constexpr (C::kOutBytes == 2) {
                        uint16_t* s16 = reinterpret_cast<uint16_t*>(stg);
#pragma unroll
                        for (int j = 0; j < CC; j += 2) {
                            const float lo = __uint_as_float(r[j]) * scale, hi = __uint_as_float(r[j + 1]) * scale;
                            const uint32_t v = C::kOut == Out::BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
                            s16[j * 128 + row_in_half] = (uint16_t)(v & 0xFFFFu);
                            s16[(j + 1) * 128 + row_in_half] = (uint16_t)(v >> 16);
                        }
                    } else {
                        uint32_t* s32 = reinterpret_cast<uint32_t*>(stg);
#pragma unroll
                        for (int j = 0; j < CC; ++j) s32[j * 128 + row_in_half] = r[j];
                    }
                    fence_proxy_async_smem();
                    named_sync(1, 128);
                    if (issuer && m0 < p.M && n_base + CC * c < p.N) {  // skip boxes wholly outside D
                        tma_store_2d(&tmD, stg, m0, n_base + CC * c);
                        bulk_commit();
                    }
                    ++chunk_seq;
                } else if (m < p.M) {
                    const size_t ldd = (size_t)p.M;
#pragma unroll
                    for (int j = 0; j < CC; j += 2) {
                        const int n = n_base + CC * c + j;
                        if constexpr (C::kOutBytes == 2) {
                            uint16_t* drow = static_cast<uint16_t*>(p.D) + m;
                            const float lo = __uint_as_float(r[j]) * scale, hi = __uint_as_float(r[j + 1]) * scale;
                            const uint32_t v = C::kOut == Out::BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
                            if (n < p.N) drow[(size_t)n * ldd] = (uint16_t)(v & 0xFFFFu);
                            if (n + 1 < p.N) drow[(size_t)(n + 1) * ldd] = (uint16_t)(v >> 16);
                        } else {
                            uint32_t* drow = static_cast<uint32_t*>(p.D) + m;
                            if (n < p.N) drow[(size_t)n * ldd] = r[j];
                            if (n + 1 < p.N) drow[(size_t)(n + 1) * ldd] = r[j + 1];
                        }
                    }
                }
                if (c + 1 < nch) tmem_ld_wait();
            };
            uint32_t ra[CC], rb[CC];
            tmem_ld_cols<CC>(t_addr, ra);
            tmem_ld_wait();
#pragma unroll 1
            for (int c = 0; c < nch; c += 2) {  // nch is even
                chunk(c, ra, rb);
                chunk(c + 1, rb, ra);
            }
            }
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (issuer) bulk_wait<0>();  // every store of D has completed
    }

    // Warps 0 and 1 arrive here diverged (one lane ran the producer or MMA
    // loop): reconverge them, then the cluster-wide barrier holds the TMEM
    // release until every epilogue warp of both CTAs has finished reading it.
    __syncwarp();
    tc_fence_before();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, G::kTmemCols);
    }
}

template <int BN>
constexpr int smem_bytes() {
    return (int)sizeof(Smem<BN>) + 1024;
}

// 2-D tensor map over `rows` rows of `row_bytes` bytes (pitch `pitch`),
// addressed in bytes, box 128 bytes x box_rows, 128-byte swizzle. Used for
// every operand whatever its element type: TMA moves bytes, the MMA's
// instruction descriptor gives them their type.
static int encode_operand(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows,
                          CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    return encode_tmap_2d_u8(map, base, row_bytes, rows, row_bytes, 128, box_rows, swizzle);
}

template <class C, int BN>
static int launch_bn(const void* A, const void* B, void* D, int M, int N, int K, cudaStream_t stream,
                     const float* scale_a, const float* scale_b, bool accumulate) {
    using G = Geom<BN>;
    constexpr int kSmemBytes = smem_bytes<BN>();
    DeviceInfo d;
    int st = require_sm100(&d);
    if (st != GPLK_STATUS_OK) return st;
    if (kSmemBytes > d.max_smem_optin) return GPLK_STATUS_UNSUPPORTED;
    static thread_local uint64_t configured = 0;  // bit per device
    static int capacity[64] = {0};                // clusters resident at once, per device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GPLK_STATUS_CUDA_ERROR;
    if (!(configured & (1ull << dev))) {
        if (cudaFuncSetAttribute(gemm_pair_kernel<C, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSmemBytes) != cudaSuccess)
            return GPLK_STATUS_LAUNCH_FAIL;
        configured |= 1ull << dev;
    }
    if (capacity[dev] == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(d.sm_count & ~1), 1, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = (size_t)kSmemBytes;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<C, BN>, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = d.sm_count / 2;
        }
        capacity[dev] = n;
    }
    CUtensorMap tmA, tmB, tmD;
    if constexpr (C::kAKMajor) {
        // A K-major (TN): M rows of K elements, boxes of 128 bytes (K) x 128 rows (M).
        st = encode_operand(&tmA, A, (uint64_t)K * C::kInBytes, (uint64_t)M, 128);
    } else {
        // A column-major M x K: K rows of M elements, boxes of kRowElems (M) x kRowElems (K).
        st = encode_operand(&tmA, A, (uint64_t)M * C::kInBytes, (uint64_t)K, (uint32_t)C::kRowElems,
                            C::kA32BAtoms ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (st != GPLK_STATUS_OK) return st;
    // B column-major K x N: N rows of K elements, boxes of 128 bytes (K) x
    // kBBox = 64 rows (N); a CTA's BN / 2 rows of a tile take BN / 128 boxes.
    st = encode_operand(&tmB, B, (uint64_t)K * C::kInBytes, (uint64_t)N, (uint32_t)G::kBBox);
    if (st != GPLK_STATUS_OK) return st;
    Params p;
    memset(&p, 0, sizeof(p));
    p.D = D;
    p.M = M;
    p.N = N;
    p.K = K;
    p.m_tiles = (M + 255) / 256;
    p.n_tiles = (N + BN - 1) / BN;
    p.scale_a = scale_a;
    p.scale_b = scale_b;
    p.accumulate = accumulate ? 1 : 0;
    {
        // As many pair-tiles per raster group as keep the group's A panels
        // within the budget, between 8 and 16: 16 for FP8 / INT8 at K = 8192,
        // 8 for BF16 / FP16 / TF32. Measured DRAM reads per 8192^3 launch
        // (ncu): BF16 1.44 / 1.08 / 1.22 GB with groups of 4 / 8 / 16, TF32
        // 4.31 / 2.98 / 2.28 GB with groups of 2 / 4 / 8; with odd groups
        // walking N backwards, BF16 1.02 GB and TF32 2.20 GB at 8.
        const size_t panel = (size_t)256 * (size_t)K * (size_t)C::kInBytes;
        const size_t g = panel ? kPanelBudget / panel : (size_t)kMaxGroupM;
        p.group_m = (int)(g < (size_t)kMinGroupM ? (size_t)kMinGroupM : g > (size_t)kMaxGroupM ? (size_t)kMaxGroupM : g);
    }
    p.k_stages = (K + C::kRowElems * kSlabs - 1) / (C::kRowElems * kSlabs);
    memset(&tmD, 0, sizeof(tmD));
    p.tma_store = ((size_t)M * C::kOutBytes) % 16 == 0 && aligned16(D);
    p.frag_store = (C::kOutBytes == 2 && p.tma_store && !accumulate) ? 1 : 0;
    if (p.tma_store) {
        // 2-byte D at beta = 0: two 128-byte-swizzled boxes of 64 rows per
        // 32-column chunk (stmatrix staging); otherwise [column][row] chunks
        // of 128 rows.
        st = p.frag_store
                 ? encode_tmap_2d_u16(&tmD, D, (uint64_t)M, (uint64_t)N, (uint64_t)M * 2, 64, C::kChunkCols,
                                      CU_TENSOR_MAP_SWIZZLE_128B)
             : C::kOutBytes == 2
                 ? encode_tmap_2d_u16(&tmD, D, (uint64_t)M, (uint64_t)N, (uint64_t)M * 2, 128, C::kChunkCols)
                 : encode_tmap_2d_u32(&tmD, D, (uint64_t)M, (uint64_t)N, (uint64_t)M * 4, 128, C::kChunkCols);
        if (st != GPLK_STATUS_OK) return st;
    }
    const int tiles = p.m_tiles * p.n_tiles;
    const int clusters = capacity[dev] < tiles ? capacity[dev] : tiles;
    // A last wave of 256 x 256 tiles that would leave at least half the
    // pairs idle runs as 256 x 128 halves, one per pair (4096^3: 256 tiles
    // = 3 waves of 74 + 34, run as 3 waves + 68 halves). Each half loads
    // only its columns of B and issues N = 128 MMAs; every output element
    // still sums its K-blocks in the same order.
    const int rem = tiles % clusters;
    p.full_items = tiles;
    p.num_items = tiles;
    if (BN == 256 && tiles > clusters && rem > 0 && 2 * rem <= clusters && N % 256 == 0) {
        p.full_items = tiles - rem;
        p.num_items = p.full_items + 2 * rem;
    }
    return launch_status(launch_pdl(gemm_pair_kernel<C, BN>, dim3(2 * clusters), dim3(kThreads), kSmemBytes,
                                    stream, tmA, tmB, tmD, p));
}

// Tile plan of one GEMM: the CTA-pair kernel with 256 x 256 or 256 x 128
// tiles, or, where the caller has one (FP8, `single`), the single-CTA kernel
// with 128 x 256 / 128 / 64 tiles. Problems that give the 256 x 256 pair
// tiles at least one full wave keep them (fewest operand bytes per FLOP).
// A smaller problem takes the candidate whose tiles, in a single wave, leave
// the fewest SMs idle; at equal fill the single-CTA tile, then the wider one.
// Measured with CUDA-graph replays on B200 (TFLOP/s, FP8 / BF16):
//   1024^3  1-CTA 128x64 473 (pair 256x256 241) / pair 256x128 247 (256x256 195)
//   1536^3  1-CTA 128x128 1116 (pair 256x128 844) / pair 256x128 630 (256x256 536)
//   2048^3  1-CTA 128x256 1609 (pair 256x256 1421) / pair 256x256 995 (256x128 793)
//   3072^3  pair 256x256 2195 (1-CTA 128x256 2153) / pair 256x256 1309
// (With its TMEM loads pipelined, the single-CTA FP8 kernel then measured
// 501 / 1203 / 1648 at 1024 / 1536 / 2048^3, widening its lead there.)
// Pair tiles 256 x 64 were never the fastest (FP8 1024^3: 324) and are not built.
struct TilePlan {
    bool pair;
    int bn;
};

static TilePlan tile_plan(int M, int N, int K, int sm_count, bool single) {
    (void)K;
    const long pair_slots = sm_count / 2;
    const bool pair_ok = M > 128 || !single;
    if (pair_ok && (long)((M + 255) / 256) * ((N + 255) / 256) >= pair_slots) return {true, 256};
    struct Cand {
        bool pair;
        int bn;
    };
    // In order of preference at equal fill.
    const Cand cands[5] = {{false, 256}, {true, 256}, {false, 128}, {true, 128}, {false, 64}};
    TilePlan best{pair_ok, pair_ok ? 256 : 64};
    double best_fill = -1.0;
    for (const Cand& c : cands) {
        if (c.pair ? !pair_ok : !single) continue;
        const long tiles = (long)((M + (c.pair ? 255 : 127)) / (c.pair ? 256 : 128)) * ((N + c.bn - 1) / c.bn);
        const long slots = c.pair ? pair_slots : sm_count;
        if (tiles > slots) continue;  // more than one wave
        const double fill = (double)tiles / (double)slots;
        if (fill > best_fill + 1e-9) {
            best_fill = fill;
            best = {c.pair, c.bn};
        }
    }
    return best;
}

template <class C>
static int launch_pair(int bn, const void* A, const void* B, void* D, int M, int N, int K, cudaStream_t stream,
                       const float* scale_a = nullptr, const float* scale_b = nullptr, bool accumulate = false) {
    if (bn == 128) return launch_bn<C, 128>(A, B, D, M, N, K, stream, scale_a, scale_b, accumulate);
    return launch_bn<C, 256>(A, B, D, M, N, K, stream, scale_a, scale_b, accumulate);
}

// Arguments shared by the four entry points. Operand pitches must be
// multiples of 16 bytes for TMA: M and K multiples of 16 / element size.
template <class C>
static int checked_launch(const void* A, const void* B, void* D, int M, int N, int K, cudaStream_t stream,
                          bool accumulate = false) {
    if (M < 0 || N < 0 || K < 0) return GPLK_STATUS_BAD_ARG;
    if (M == 0 || N == 0) return GPLK_STATUS_OK;
    constexpr int align = 16 / C::kInBytes;
    if (K == 0 || M % align != 0 || K % align != 0) return GPLK_STATUS_BAD_ARG;
    if (!A || !B || !D || !aligned16(A) || !aligned16(B)) return GPLK_STATUS_BAD_ARG;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != GPLK_STATUS_OK) return st;
    const TilePlan plan = tile_plan(M, N, K, d.sm_count, false);
    return launch_pair<C>(plan.bn, A, B, D, M, N, K, stream, nullptr, nullptr, accumulate);
}

}  // namespace pair
}  // namespace gplk

extern "C" int gplk_gemm_bf16_nn(const uint16_t* A, const uint16_t* B, uint16_t* D, int M, int N, int K,
                                 cudaStream_t stream) {
    return gplk::pair::checked_launch<gplk::pair::CfgBF16>(A, B, D, M, N, K, stream);
}

extern "C" int gplk_gemm_f16_nn(const uint16_t* A, const uint16_t* B, uint16_t* D, int M, int N, int K,
                                cudaStream_t stream) {
    return gplk::pair::checked_launch<gplk::pair::CfgF16>(A, B, D, M, N, K, stream);
}

extern "C" int gplk_gemm_tf32_nn(const float* A, const float* B, float* D, int M, int N, int K,
                                 cudaStream_t stream) {
    return gplk::pair::checked_launch<gplk::pair::CfgTF32>(A, B, D, M, N, K, stream);
}

extern "C" int gplk_gemm_i8_nn(const int8_t* A, const int8_t* B, int32_t* D, int M, int N, int K,
                               cudaStream_t stream) {
    return gplk::pair::checked_launch<gplk::pair::CfgI8>(A, B, D, M, N, K, stream);
}

extern "C" int gplk_gemm_bf16_nn_acc(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K,
                                     cudaStream_t stream) {
    return gplk::pair::checked_launch<gplk::pair::CfgBF16>(A, B, C, M, N, K, stream, true);
}

extern "C" int gplk_gemm_f16_nn_acc(const uint16_t* A, const uint16_t* B, uint16_t* C, int M, int N, int K,
                                    cudaStream_t stream) {
    return gplk::pair::checked_launch<gplk::pair::CfgF16>(A, B, C, M, N, K, stream, true);
}

extern "C" int gplk_gemm_tf32_nn_acc(const float* A, const float* B, float* C, int M, int N, int K,
                                     cudaStream_t stream) {
    return gplk::pair::checked_launch<gplk::pair::CfgTF32>(A, B, C, M, N, K, stream, true);
}

extern "C" int gplk_gemm_i8_nn_acc(const int8_t* A, const int8_t* B, int32_t* C, int M, int N, int K,
                                   cudaStream_t stream) {
    return gplk::pair::checked_launch<gplk::pair::CfgI8>(A, B, C, M, N, K, stream, true);
}
