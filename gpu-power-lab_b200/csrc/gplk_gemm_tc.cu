// gplk_gemm_tc.cu - tcgen05 GEMMs for the narrow formats of the GEMM ladder:
//   FP8   E4M3 x E4M3, per-tensor FP32 scales           (kind::f8f6f4)
//   NVFP4 E2M1 x E2M1, UE4M3 scale per 16 K-elements     (kind::mxf4nvf4.block16)
// both with FP32 accumulation in TMEM and BF16 output, in cuBLASLt's TN
// convention (A and B K-major, D column-major M x N). FP8 problems go to
// this kernel or to the CTA-pair kernel of gplk_gemm_pair.cu by
// pair::tile_plan.
//
// One persistent CTA per SM walks output tiles of 128 x BN in a grouped
// (L2-friendly) order, launched with programmatic stream serialisation (its
// set-up overlaps the previous GEMM on the stream). BN is 256 for NVFP4;
// FP8 takes BN = 256, 128 or 64 as pair::tile_plan decides (1024^3 has 16
// CTA-pair tiles of 256 x 256 but 128 tiles of 128 x 64). NVFP4 runs a
// last wave that would leave half the CTAs idle as 128 x 128 half tiles,
// one per CTA (work items, item_tile). Warp roles:
//   warp 0      TMA producer: 2-D tiled loads of A (128 rows) and B (BN
//               rows; for NVFP4 in 128-row boxes, one per half), 128 bytes of
//               K per stage with 128-byte swizzle, into a STAGES-deep
//               shared-memory ring; NVFP4 adds 1-D bulk copies of the
//               stage's scale-factor blocks. No cluster multicast.
//   warp 1      owns TMEM; one thread issues the MMAs (4 per stage: K = 32
//               FP8 or 64 FP4 elements per instruction) and, for NVFP4,
//               the shared->TMEM copies of the scale factors first.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, scale, BF16, staged
//               in shared memory and written by TMA stores (plain stores when
//               D's rows are not 16-byte multiples). Warp w reads TMEM lanes
//               32*(w%4)..+31 (= tile rows).
// FP8 double-buffers the accumulator (2 x BN TMEM columns) so the epilogue of
// one tile overlaps the main loop of the next. NVFP4
// needs TMEM for per-stage scale factors, so it keeps one accumulator and
// drains it into registers before storing, releasing TMEM early.
// Every mbarrier wait is bounded; on timeout the kernel records
// GPLK_STATUS_DEVICE_TIMEOUT, drains outstanding copies and MMAs, frees TMEM
// and returns.
#include <cstring>

#include "gplk_ptx.cuh"

namespace gplk {
namespace gemm_tc {

constexpr int BM = 128;
constexpr int BK_BYTES = 128;  // one 128-byte swizzle row of K per stage
constexpr int A_STAGE = BM * BK_BYTES;   // 16 KiB
constexpr int SFA_STAGE = 4 * 512;       // 4 K-blocks of 128 rows x 4 scales
constexpr int SFB_STAGE = 8 * 512;       // 2 row-halves x 4 K-blocks
constexpr int kThreads = 192;
constexpr int kGroupM = 8;               // tile raster group along M

template <bool NVF4, int BN = 256>
struct Traits {
    static_assert(BN == 256 || (!NVF4 && (BN == 128 || BN == 64)), "tile width");
    static constexpr int kBN = BN;
    static constexpr int kBStage = BN * BK_BYTES;  // 32 / 16 / 8 KiB
    // Narrower tiles have smaller stages: a deeper ring in the same memory.
    static constexpr int kStages = BN == 256 ? 4 : 6;
    static constexpr int kStageBytes = A_STAGE + kBStage + (NVF4 ? SFA_STAGE + SFB_STAGE : 0);
    static constexpr int kAccBufs = NVF4 ? 1 : 2;
    static constexpr uint32_t kTmemCols = NVF4 ? 512u : (uint32_t)(2 * BN);
    // TMEM column map. Accumulators first; NVFP4 scale factors after them,
    // one 48-column slot per stage (16 for A, 32 for B).
    static constexpr uint32_t kSfCol0 = 256;
    static constexpr uint32_t kSfColsPerStage = 48;
    static_assert(!NVF4 || kSfCol0 + kStages * kSfColsPerStage <= kTmemCols, "TMEM budget");
};

template <bool NVF4, int BN = 256>
struct __align__(1024) Smem {
    uint8_t stage[Traits<NVF4, BN>::kStages][Traits<NVF4, BN>::kStageBytes];
    // Epilogue staging, 8 KiB BF16 chunks of 128 rows x 32 columns: one for
    // NVFP4 ([column][row]; its ring leaves room for one), two for FP8 (each
    // two 128-byte-swizzled TMA boxes of 64 rows x 32 columns).
    uint8_t out_stage[NVF4 ? 1 : 2][128 * 32 * 2];
    uint64_t full[Traits<NVF4, BN>::kStages];
    uint64_t empty[Traits<NVF4, BN>::kStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
    int epi_fail;
};

struct Params {
    uint16_t* D;
    int group_m;           // raster group along M (tiles)
    const uint8_t* sfa;  // NVFP4 only
    const uint8_t* sfb;
    const float* scale_a;  // FP8: per-tensor scales; NVFP4: scale_a = alpha
    const float* scale_b;
    int M, N, K;           // K in elements
    int m_tiles, n_tiles, k_stages;
    int sf_kblocks4;       // NVFP4: ceil(K / 64) = 512-byte blocks per 128 rows
    int sf_row_blocks_b;   // NVFP4: ceil(N / 128) row blocks in SFB
    int tma_store;         // write D with TMA stores (M % 8 == 0, 16-byte aligned D)
    // Work items: items below full_items are whole tiles (item = tile);
    // the rest split the last wave's tiles into 128-column halves (NVFP4).
    int full_items, num_items;
};

// Work item -> tile and column half (-1: the whole 128 x BN tile).
__device__ __forceinline__ int item_tile(const Params& p, int item, int& half) {
    if (item < p.full_items) {
        half = -1;
        return item;
    }
    const int u = item - p.full_items;
    half = u & 1;
    return p.full_items + (u >> 1);
}

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& mt, int& nt,
                                            int group_m = kGroupM) {
    const int per_group = group_m * n_tiles;
    const int group = t / per_group;
    const int first_m = group * group_m;
    const int gsize = min(m_tiles - first_m, group_m);
    const int r = t % per_group;
    mt = first_m + r % gsize;
    nt = r / gsize;
}

template <bool NVF4, int BN = 256>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmD, const Params p) {
    using TR = Traits<NVF4, BN>;
    constexpr int S = TR::kStages;
    constexpr int B_STAGE = TR::kBStage;
    extern __shared__ uint8_t smem_raw[];
    Smem<NVF4, BN>& sm = *reinterpret_cast<Smem<NVF4, BN>*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);

    const uint32_t warp = warp_id_uniform();
    const uint32_t lane = lane_id();

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&sm.full[i], 1);
            mbar_init(&sm.empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.acc_full[i], 1);
            mbar_init(&sm.acc_empty[i], 4);
        }
        mbar_init(&sm.drain, 1);
        sm.abort = 0;
        sm.epi_fail = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(&sm.tmem_base, TR::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    // Launched with programmatic stream serialisation: the set-up above may
    // overlap the previous kernel's tail; nothing below touches global
    // memory before that kernel has completed. The next GEMM on the stream
    // may then be launched into SMs as they free up.
    pdl_wait();
    pdl_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, issued_parity = 0;  // for the abort drain
            bool ok = true;
            for (int it = blockIdx.x; it < p.num_items && ok; it += gridDim.x) {
                int half;
                const int t = item_tile(p, it, half);
                int mt, nt;
                tile_coords(t, p.m_tiles, p.n_tiles, mt, nt, p.group_m);
                for (int kb = 0; kb < p.k_stages; ++kb) {
                    if (!mbar_wait(&sm.empty[stage], phase ^ 1u, &sm.abort, 0x0201)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = sm.stage[stage];
                    if constexpr (NVF4) {
                        // B arrives in 128-row boxes: both for a whole tile, the
                        // item's own half (into the first half slot) otherwise.
                        // The A stage covers K-blocks 4*kb .. 4*kb+3 of row block
                        // mt (2 KiB contiguous); B's scales are row blocks 2*nt
                        // and 2*nt + 1, or the half's own one.
                        const size_t blk = (size_t)p.sf_kblocks4;
                        const uint8_t* sa = p.sfa + ((size_t)mt * blk + (size_t)kb * 4) * 512;
                        uint8_t* dsf = st + A_STAGE + B_STAGE;
                        if (half < 0) {
                            mbar_arrive_expect_tx(&sm.full[stage], TR::kStageBytes);
                            tma_load_2d(st, &tmA, &sm.full[stage], kb * BK_BYTES, mt * BM);
                            tma_load_2d(st + A_STAGE, &tmB, &sm.full[stage], kb * BK_BYTES, nt * BN);
                            tma_load_2d(st + A_STAGE + B_STAGE / 2, &tmB, &sm.full[stage], kb * BK_BYTES,
                                        nt * BN + 128);
                            const uint8_t* sb0 = p.sfb + ((size_t)(2 * nt) * blk + (size_t)kb * 4) * 512;
                            // A last tile with N % 256 <= 128 has no second row
                            // block; its B rows are zero-filled by TMA and never
                            // stored, so any in-bounds scale bytes will do.
                            const int nb1 = (2 * nt + 1 < p.sf_row_blocks_b) ? 2 * nt + 1 : 2 * nt;
                            const uint8_t* sb1 = p.sfb + ((size_t)nb1 * blk + (size_t)kb * 4) * 512;
                            bulk_load(dsf, sa, SFA_STAGE, &sm.full[stage]);
                            bulk_load(dsf + SFA_STAGE, sb0, SFB_STAGE / 2, &sm.full[stage]);
                            bulk_load(dsf + SFA_STAGE + SFB_STAGE / 2, sb1, SFB_STAGE / 2, &sm.full[stage]);
                        } else {
                            mbar_arrive_expect_tx(&sm.full[stage],
                                                  A_STAGE + B_STAGE / 2 + SFA_STAGE + SFB_STAGE / 2);
                            tma_load_2d(st, &tmA, &sm.full[stage], kb * BK_BYTES, mt * BM);
                            tma_load_2d(st + A_STAGE, &tmB, &sm.full[stage], kb * BK_BYTES,
                                        nt * BN + 128 * half);
                            const uint8_t* sbh =
                                p.sfb + ((size_t)(2 * nt + half) * blk + (size_t)kb * 4) * 512;
                            bulk_load(dsf, sa, SFA_STAGE, &sm.full[stage]);
                            bulk_load(dsf + SFA_STAGE, sbh, SFB_STAGE / 2, &sm.full[stage]);
                        }
                    } else {
                        mbar_arrive_expect_tx(&sm.full[stage], TR::kStageBytes);
                        tma_load_2d(st, &tmA, &sm.full[stage], kb * BK_BYTES, mt * BM);
                        tma_load_2d(st + A_STAGE, &tmB, &sm.full[stage], kb * BK_BYTES, nt * BN);
                    }
                    issued_mask |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok || sm.abort) {
                // Drain: every issued copy must land before the block exits.
                int dummy = 0;
                for (int s2 = 0; s2 < S; ++s2)
                    if (issued_mask & (1u << s2))
                        mbar_wait(&sm.full[s2], (issued_parity >> s2) & 1u, &dummy, 0x0202,
                                  100000000ull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc_full = NVF4 ? idesc_nvf4(BM, BN) : idesc_e4m3_f32(BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int it = blockIdx.x; it < p.num_items && ok; it += gridDim.x) {
                int half;
                (void)item_tile(p, it, half);
                // A half item multiplies its 128 B rows (loaded into the first
                // half slot) into accumulator columns 0..127, with N = 128.
                const uint32_t idesc = (NVF4 && half >= 0) ? idesc_nvf4(BM, 128) : idesc_full;
                const int sfb_halves = half < 0 ? 2 : 1;
                if (!mbar_wait(&sm.acc_empty[acc], acc_phase ^ 1u, &sm.abort, 0x0211)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)acc * (uint32_t)BN;
                for (int kb = 0; kb < p.k_stages; ++kb) {
                    if (!mbar_wait(&sm.full[stage], phase, &sm.abort, 0x0212)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sm.stage[stage]);
                    const uint32_t b_addr = a_addr + A_STAGE;
                    if constexpr (NVF4) {
                        const uint32_t sf_addr = b_addr + B_STAGE;
                        const uint32_t sf_col = tmem + TR::kSfCol0 + (uint32_t)stage * TR::kSfColsPerStage;
                        // A: K-block j -> 4 columns at sf_col + 4j.
                        // B: K-block j, row half h -> 4 columns at sf_col + 16 + 8j + 4h.
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            tmem_cp_32x128b_warpx4(sf_col + 4 * j, smem_desc(sf_addr + 512 * j, 0, 128, 0));
#pragma unroll
                            for (int h = 0; h < 2; ++h)
                                if (h < sfb_halves)
                                    tmem_cp_32x128b_warpx4(
                                        sf_col + 16 + 8 * j + 4 * h,
                                        smem_desc(sf_addr + SFA_STAGE + h * (SFB_STAGE / 2) + 512 * j, 0, 128, 0));
                        }
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            mma_nvf4(d_tmem, desc_kmajor_sw128(a_addr + 32 * j),
                                     desc_kmajor_sw128(b_addr + 32 * j), idesc, sf_col + 4 * j,
                                     sf_col + 16 + 8 * j, (kb | j) != 0);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            mma_f8f6f4(d_tmem, desc_kmajor_sw128(a_addr + 32 * j),
                                       desc_kmajor_sw128(b_addr + 32 * j), idesc, (kb | j) != 0);
                        }
                    }
                    tc_commit(&sm.empty[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(&sm.acc_full[acc]);
                if (++acc == TR::kAccBufs) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            // Every MMA issued by this thread completes before TMEM is freed.
            tc_commit(&sm.drain);
            int dummy = 0;
            mbar_wait(&sm.drain, 0, &dummy, 0x0213, 100000000ull);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const uint32_t quarter = warp & 3u;  // TMEM lanes 32*quarter .. +31
        const int row_in_tile = (int)(quarter * 32 + lane);
        const float scale = NVF4 ? __ldg(p.scale_a) : __ldg(p.scale_a) * __ldg(p.scale_b);
        int acc = 0;
        uint32_t acc_phase = 0;
        uint32_t chunk_seq = 0;  // FP8 staging buffer rotation
        for (int it = blockIdx.x; it < p.num_items; it += gridDim.x) {
            int half;
            const int t = item_tile(p, it, half);
            int mt, nt;
            tile_coords(t, p.m_tiles, p.n_tiles, mt, nt, p.group_m);
            // All four epilogue warps leave together if any of them gave up
            // (the staged store path synchronises them with a named barrier).
            if (!mbar_wait_sleepy(&sm.acc_full[acc], acc_phase, &sm.abort, 0x0221, false)) sm.epi_fail = 1;
            named_sync(1, 128);
            if (*(volatile int*)&sm.epi_fail) break;
            tc_fence_after();
            const int m = mt * BM + row_in_tile;
            const int n_base = nt * BN + (half > 0 ? 128 : 0);
            const uint32_t t_addr = tmem + ((quarter * 32u) << 16) + (uint32_t)acc * (uint32_t)BN;
            uint16_t* drow = p.D + m;  // column-major: D[m + n * M]
            const size_t ldd = (size_t)p.M;
            if constexpr (NVF4) {
                // Drain the accumulator's columns (256, or 128 for a half
                // item) to registers, release TMEM, then store. With TMA
                // stores the drain reads 16-lane mma fragments
                // (tcgen05.ld.16x256b, as the FP8 epilogue below) for stmatrix
                // staging; packed[16c + 4k + i] then holds 8 x 8 block i of
                // column group k of chunk c. Plain stores keep this thread's
                // row: packed[16c + j] = columns 32c + 2j, +1.
                const int nch = half < 0 ? 8 : 4;  // 32-column chunks
                uint32_t packed[128];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    if (c >= nch) continue;
                    if (p.tma_store) {
                        uint32_t x[2][16];
                        const uint32_t lanes0 = tmem + ((quarter * 32u) << 16) + 32u * (uint32_t)c;
                        tmem_ld_16x256b_x4(lanes0, x[0]);
                        tmem_ld_16x256b_x4(lanes0 + (16u << 16), x[1]);
                        tmem_ld_wait();
#pragma unroll
                        for (int k = 0; k < 4; ++k)
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const int h = i >> 1, e = 4 * k + 2 * (i & 1);
                                packed[c * 16 + 4 * k + i] = pack_bf16x2(__uint_as_float(x[h][e]) * scale,
                                                                         __uint_as_float(x[h][e + 1]) * scale);
                            }
                    } else {
                        uint32_t r[32];
                        tmem_ld_32x32b_x32(t_addr + 32u * c, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            packed[c * 16 + j] = pack_bf16x2(__uint_as_float(r[2 * j]) * scale,
                                                             __uint_as_float(r[2 * j + 1]) * scale);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.acc_empty[acc]);
                if (p.tma_store) {
                    // One 8 KiB staging buffer (two 128-byte-swizzled boxes of
                    // 64 rows x 32 columns): wait for the previous store to
                    // read it, fill it with stmatrix, store.
                    const bool issuer = warp == 2 && lane == 0;
                    const int m0 = mt * BM;
                    const int r0 = (int)quarter * 32 + 8 * (int)(lane >> 3);
                    const uint32_t jr = lane & 7u;
                    const uint32_t sbase = smem_u32(sm.out_stage[0]) + (uint32_t)(r0 >> 6) * 4096u;
                    const uint32_t chk = (uint32_t)((r0 & 63) >> 3);
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        if (c >= nch) continue;  // uniform over the four warps
                        if (issuer) bulk_wait_read<0>();
                        named_sync(1, 128);
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint32_t cc = (uint32_t)(8 * k) + jr;
                            stmatrix_x4_trans(sbase + cc * 128u + ((chk ^ (cc & 7u)) << 4), packed[c * 16 + 4 * k],
                                              packed[c * 16 + 4 * k + 1], packed[c * 16 + 4 * k + 2],
                                              packed[c * 16 + 4 * k + 3]);
                        }
                        fence_proxy_async_smem();
                        named_sync(1, 128);
                        if (issuer && n_base + 32 * c < p.N) {
                            const uint8_t* stg = sm.out_stage[0];
                            tma_store_2d(&tmD, stg, m0, n_base + 32 * c);
                            if (m0 + 64 < p.M) tma_store_2d(&tmD, stg + 4096, m0 + 64, n_base + 32 * c);
                            bulk_commit();
                        }
                    }
                } else if (m < p.M) {
#pragma unroll
                    for (int j = 0; j < 128; ++j) {
                        if (j >= 16 * nch) continue;
                        const int n = n_base + 2 * j;
                        if (n < p.N) drow[(size_t)n * ldd] = (uint16_t)(packed[j] & 0xFFFFu);
                        if (n + 1 < p.N) drow[(size_t)(n + 1) * ldd] = (uint16_t)(packed[j] >> 16);
                    }
                }
            } else if (p.tma_store) {
                // FP8 with TMA stores (M % 8 == 0, 16-byte aligned D). Per
                // 32-column chunk each warp loads its 32 rows as two 16-lane
                // tcgen05.ld.16x256b.x4, whose registers are mma fragments:
                // thread t holds rows t/4 and t/4 + 8 at columns 2(t%4), +1 of
                // every 8-column group. Scaled and rounded to BF16 pairs they
                // go to shared memory through stmatrix .trans (each 8 x 8 block
                // lands as 8 columns of 8 consecutive rows, 16 bytes each) in
                // the 128-byte-swizzled layout of two 64-row x 32-column TMA
                // store boxes, so a warp's 2 KiB take 16 conflict-free
                // wavefronts (column-major 2-byte stores took 32 and 32
                // instructions). The loads of chunk c + 1 are issued before
                // chunk c is stored; the accumulator is released once its last
                // chunk is in registers. Two staging buffers: the stores of
                // one chunk overlap the staging of the next.
                const bool issuer = warp == 2 && lane == 0;
                const int m0 = mt * BM;
                constexpr int NC = BN / 32;
                const uint32_t lanes0 = tmem + ((quarter * 32u) << 16) + (uint32_t)acc * (uint32_t)BN;
                const uint32_t lanes1 = lanes0 + (16u << 16);
                // stmatrix: thread 8m + j gives the address of row j (a D
                // column) of matrix m, which holds tile rows r0 .. r0 + 7.
                const int r0 = (int)quarter * 32 + 8 * (int)(lane >> 3);
                const uint32_t jr = lane & 7u;
                const uint32_t box_off = (uint32_t)(r0 >> 6) * 4096u;  // rows 64..127: second box
                const uint32_t chk = (uint32_t)((r0 & 63) >> 3);         // 16-byte unit within a 128-byte line
                uint32_t x[2][2][16];
                tmem_ld_16x256b_x4(lanes0, x[0][0]);
                tmem_ld_16x256b_x4(lanes1, x[0][1]);
                tmem_ld_wait();
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const int cur = c & 1;
                    if (c + 1 < NC) {
                        tmem_ld_16x256b_x4(lanes0 + 32u * (uint32_t)(c + 1), x[cur ^ 1][0]);
                        tmem_ld_16x256b_x4(lanes1 + 32u * (uint32_t)(c + 1), x[cur ^ 1][1]);
                    } else {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&sm.acc_empty[acc]);
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
                            return pack_bf16x2(__uint_as_float(x[cur][h][i]) * scale,
                                               __uint_as_float(x[cur][h][i + 1]) * scale);
                        };
                        stmatrix_x4_trans(addr, pk(0, 4 * k), pk(0, 4 * k + 2), pk(1, 4 * k), pk(1, 4 * k + 2));
                    }
                    fence_proxy_async_smem();
                    named_sync(1, 128);
                    if (issuer && n_base + 32 * c < p.N) {
                        tma_store_2d(&tmD, stg, m0, n_base + 32 * c);
                        if (m0 + 64 < p.M) tma_store_2d(&tmD, stg + 4096, m0 + 64, n_base + 32 * c);
                        bulk_commit();
                    }
                    ++chunk_seq;
                    if (c + 1 < NC) tmem_ld_wait();
                }
            } else {
                // FP8 with plain stores (D's rows not 16-byte multiples): per
                // 32-column chunk, tcgen05.ld of this thread's row, scale,
                // BF16, stored column by column; the load of chunk c + 1 is
                // issued before chunk c is stored.
                constexpr int NC = BN / 32;
                uint32_t rr[2][32];
                tmem_ld_32x32b_x32(t_addr, rr[0]);
                tmem_ld_wait();
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const int cur = c & 1;
                    if (c + 1 < NC) {
                        tmem_ld_32x32b_x32(t_addr + 32u * (c + 1), rr[cur ^ 1]);
                    } else {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&sm.acc_empty[acc]);
                    }
                    if (m < p.M) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const uint32_t pkd = pack_bf16x2(__uint_as_float(rr[cur][2 * j]) * scale,
                                                             __uint_as_float(rr[cur][2 * j + 1]) * scale);
                            const int n = n_base + 32 * c + 2 * j;
                            if (n < p.N) drow[(size_t)n * ldd] = (uint16_t)(pkd & 0xFFFFu);
                            if (n + 1 < p.N) drow[(size_t)(n + 1) * ldd] = (uint16_t)(pkd >> 16);
                        }
                    }
                    if (c + 1 < NC) tmem_ld_wait();
                }
            }
            if (++acc == TR::kAccBufs) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (p.tma_store && warp == 2 && lane == 0) bulk_wait<0>();  // every store of D has completed
    }

    // Warps 0 and 1 arrive here diverged (one lane ran the producer or MMA
    // loop): reconverge them, then the block-wide barrier holds the TMEM
    // release until every epilogue warp has finished reading it.
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TR::kTmemCols);
    }
}


template <bool NVF4, int BN>
static int smem_bytes() {
    return (int)sizeof(Smem<NVF4, BN>) + 1024;
}

template <bool NVF4, int BN = 256>
static int launch(const uint8_t* A, const uint8_t* B, const uint8_t* SFA, const uint8_t* SFB,
                  uint16_t* D, int M, int N, int K, const float* sa, const float* sb,
                  cudaStream_t stream) {
    DeviceInfo d;
    int st = require_sm100(&d);
    if (st != GPLK_STATUS_OK) return st;
    const int smem = smem_bytes<NVF4, BN>();
    if (smem > d.max_smem_optin) return GPLK_STATUS_UNSUPPORTED;
    static thread_local uint64_t configured = 0;  // bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1ull << dev))) {
        if (cudaFuncSetAttribute(gemm_tc_kernel<NVF4, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return GPLK_STATUS_LAUNCH_FAIL;
        configured |= 1ull << dev;
    }
    // Operand row length in bytes: K for E4M3, K/2 for packed E2M1.
    const uint64_t row_bytes = NVF4 ? (uint64_t)K / 2 : (uint64_t)K;
    CUtensorMap tmA, tmB;
    st = encode_tmap_2d_u8(&tmA, A, row_bytes, (uint64_t)M, row_bytes, BK_BYTES, BM);
    if (st != GPLK_STATUS_OK) return st;
    // NVFP4 loads B in 128-row boxes (two per stage for a whole tile).
    st = encode_tmap_2d_u8(&tmB, B, row_bytes, (uint64_t)N, row_bytes, BK_BYTES, NVF4 ? 128 : BN);
    if (st != GPLK_STATUS_OK) return st;

    Params p;
    memset(&p, 0, sizeof(p));
    p.D = D;
    p.sfa = SFA;
    p.sfb = SFB;
    p.scale_a = sa;
    p.scale_b = sb;
    p.M = M;
    p.N = N;
    p.K = K;
    p.m_tiles = (M + BM - 1) / BM;
    p.n_tiles = (N + BN - 1) / BN;
    p.k_stages = (int)((row_bytes + BK_BYTES - 1) / BK_BYTES);
    p.sf_kblocks4 = (K + 63) / 64;
    p.sf_row_blocks_b = (N + 127) / 128;
    // A wide raster group keeps B's row blocks in L2 across more M tiles
    // (B is re-read from DRAM once per group). NVFP4 sizes the group by the
    // A rows it keeps live, 32 MiB (the CTA-pair kernel's panel budget), and
    // at least 32 M tiles: 8192^3 then runs as one group of 64, A and B
    // each fetched once, instead of two groups whose first waves both wait
    // on A's rows in DRAM (median tile 23 300 -> 21 500 SM cycles, output
    // unchanged); 4096^3 and 16384^3 keep 32.
    if (NVF4) {
        const size_t panel = (size_t)BM * (size_t)row_bytes;  // one M tile's A rows
        const size_t g = ((size_t)32 << 20) / panel;
        p.group_m = g < 32 ? 32 : (g > (size_t)p.m_tiles ? p.m_tiles : (int)g);
    } else {
        p.group_m = kGroupM;
    }
    CUtensorMap tmD;
    memset(&tmD, 0, sizeof(tmD));
    p.tma_store = (M % 8 == 0) && aligned16(D);
    if (p.tma_store) {
        // Both stage each 32-column chunk as two 128-byte-swizzled boxes of
        // 64 rows (stmatrix staging, see the epilogues).
        st = encode_tmap_2d_u16(&tmD, D, (uint64_t)M, (uint64_t)N, (uint64_t)M * 2, 64, 32,
                                CU_TENSOR_MAP_SWIZZLE_128B);
        if (st != GPLK_STATUS_OK) return st;
    }
    const int tiles = p.m_tiles * p.n_tiles;
    const int grid = tiles < d.sm_count ? tiles : d.sm_count;
    // NVFP4: when the last wave of tiles would leave at least half the CTAs
    // idle, its tiles are split into 128-column halves, one per CTA, so the
    // wave ends in about the time of a half tile (4096^3: 512 tiles = 3
    // waves of 148 + 68, run as 3 waves + 136 halves). Every output element
    // still sums its K-blocks in the same order.
    const int rem = tiles % grid;
    p.full_items = tiles;
    p.num_items = tiles;
    if (NVF4 && tiles > grid && rem > 0 && 2 * rem <= grid && N % BN == 0) {
        p.full_items = tiles - rem;
        p.num_items = p.full_items + 2 * rem;
    }
    return launch_status(launch_pdl(gemm_tc_kernel<NVF4, BN>, dim3(grid), dim3(kThreads), (size_t)smem, stream,
                                    tmA, tmB, tmD, p));
}

}  // namespace gemm_tc
}  // namespace gplk

extern "C" int gplk_gemm_fp8_tn(const uint8_t* A, const uint8_t* B, uint16_t* D, int M, int N, int K,
                                const float* scale_a, const float* scale_b, cudaStream_t stream) {
    using namespace gplk;
    if (M < 0 || N < 0 || K < 0) return GPLK_STATUS_BAD_ARG;
    if (M == 0 || N == 0) return GPLK_STATUS_OK;
    if (K == 0 || K % 16 != 0) return GPLK_STATUS_BAD_ARG;
    if (!A || !B || !D || !scale_a || !scale_b) return GPLK_STATUS_BAD_ARG;
    if (!aligned16(A) || !aligned16(B)) return GPLK_STATUS_BAD_ARG;
    DeviceInfo d;
    const int st = current_device_info(&d);
    if (st != GPLK_STATUS_OK) return st;
    // CTA-pair tiles (256 x 256 / 128) or single-CTA tiles (128 x 256 / 128 /
    // 64), whichever fills the SMs best (pair::tile_plan).
    const pair::TilePlan plan = pair::tile_plan(M, N, K, d.sm_count, true);
    if (plan.pair) return pair::launch_pair<pair::CfgFP8>(plan.bn, A, B, D, M, N, K, stream, scale_a, scale_b);
    switch (plan.bn) {
        case 128: return gemm_tc::launch<false, 128>(A, B, nullptr, nullptr, D, M, N, K, scale_a, scale_b, stream);
        case 64: return gemm_tc::launch<false, 64>(A, B, nullptr, nullptr, D, M, N, K, scale_a, scale_b, stream);
        default: return gemm_tc::launch<false, 256>(A, B, nullptr, nullptr, D, M, N, K, scale_a, scale_b, stream);
    }
}

extern "C" size_t gplk_nvfp4_sf_bytes(int rows, int k) {
    if (rows <= 0 || k <= 0) return 0;
    const size_t row_blocks = ((size_t)rows + 127) / 128;
    const size_t k_blocks4 = ((size_t)k + 63) / 64;
    return row_blocks * k_blocks4 * 512;
}

extern "C" int gplk_gemm_nvfp4_tn(const uint8_t* A, const uint8_t* B, const uint8_t* SFA,
                                  const uint8_t* SFB, uint16_t* D, int M, int N, int K,
                                  const float* alpha, cudaStream_t stream) {
    using namespace gplk;
    if (M < 0 || N < 0 || K < 0) return GPLK_STATUS_BAD_ARG;
    if (M == 0 || N == 0) return GPLK_STATUS_OK;
    if (K == 0 || K % 256 != 0) return GPLK_STATUS_BAD_ARG;
    if (!A || !B || !SFA || !SFB || !D || !alpha) return GPLK_STATUS_BAD_ARG;
    if (!aligned16(A) || !aligned16(B) || !aligned16(SFA) || !aligned16(SFB)) return GPLK_STATUS_BAD_ARG;
    return gemm_tc::launch<true>(A, B, SFA, SFB, D, M, N, K, alpha, alpha, stream);
}
