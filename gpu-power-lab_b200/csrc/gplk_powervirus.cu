// gplk_powervirus.cu - mixed-unit power kernel for B200.
//
// One persistent block of 32 warps per SM. Warp w of block b takes the role
// role_map[(2 * w + (b & 1)) % 64], so the 32 warps of every block sample the
// 64-slot map evenly and every SM carries the whole mix at once. (The
// reference indexes the map with the global warp id, runner/src/
// workload_powervirus.cu:107-108, which hands each 8-warp block a contiguous
// slice of the map; with one block per SM that would put whole roles on
// separate SMs.)
//
// Roles (reference lines they correspond to, workload_powervirus.cu):
//   TENSOR  the block's first tensor-role warp owns 256 TMEM columns and one
//           thread issues tcgen05.mma kind::f8f6f4 128x256x32 on
//           shared-memory-resident E4M3 tiles (A 128x128, B 256x128), four
//           per K=128 tile, `inner` tiles per launch, accumulating in TMEM.
//           tcgen05 is single-thread issued, so the block's other
//           tensor-role warps have nothing to issue and park (:114-141 used
//           warp-synchronous wmma instead).
//   FMA     eight dependent FFMA chains, inner*16 steps (:142-156).
//   DRAM    TMA bulk loads (cp.async.bulk) of 8 KiB chunks of the stream
//           buffer into a 16-stage shared-memory ring owned by the block's
//           DRAM warps, inner/4 chunks per warp (the same 2 KiB x inner per
//           warp that the reference's float4 loads move, :157-170).
//   SFU, INT32, SMEM, L2, ATOMIC as the reference (:172-245).
// Nothing waits without a bound; a timeout records
// GPLK_STATUS_DEVICE_TIMEOUT and the block drains and exits.
#include "gplk_ptx.cuh"

namespace gplk {
namespace pv {

constexpr int kWarps = 32;
constexpr int kThreads = kWarps * 32;
constexpr int kSlotStride = GPLK_PV_ROLE_SLOTS / kWarps;  // 2
constexpr int kRingStages = 16;
constexpr int kChunk = 8192;
constexpr int kSmemPerWarp = 64;
constexpr uint32_t kTmemCols = 256;
constexpr int kAtomicSlots = 1024;
constexpr size_t kL2WindowBytes = 4u << 20;

struct __align__(1024) Smem {
    uint8_t mma_a[128 * 128];  // E4M3, K-major, 128-byte swizzle
    uint8_t mma_b[256 * 128];
    uint8_t ring[kRingStages][kChunk];
    float smem_role[kWarps][kSmemPerWarp];
    uint64_t ring_full[kRingStages];
    uint64_t mma_done;
    uint32_t tmem_base;
    int has_tmem;
    int abort;
    int role_count[GPLK_PV_ROLE_COUNT];
    int role_rank[kWarps];
    unsigned char role_of[kWarps];
};

struct Params {
    const unsigned char* role_map;
    const float4* stream_buf;
    size_t stream_elems;  // float4 elements
    size_t stream_chunks; // kChunk-byte chunks
    float* sink;
    uint32_t* verify_out;
    const uint8_t* mma_a;
    const uint8_t* mma_b;
    float* mma_out;
    int inner;
    uint64_t budget_ns;  // 0: fixed work; else every role continues until this long after block start
};

// Byte offset of (row, k) in a K-major tile staged with the 128-byte swizzle
// the UMMA descriptor expects: 8-row atoms of 1024 bytes, and within a row
// the 16-byte chunk index XOR (row % 8).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t k) {
    return (row >> 3) * 1024u + (row & 7u) * 128u + ((((k >> 4) ^ (row & 7u)) & 7u) << 4) + (k & 15u);
}

__device__ __forceinline__ void fill_tile(uint8_t* dst, const uint8_t* src, int rows, uint8_t pattern,
                                          uint32_t lane) {
    // src: rows x 128 bytes, row-major (K contiguous). 16 bytes per step.
    for (int i = (int)lane; i < rows * 8; i += 32) {
        const int row = i >> 3, chunk = i & 7;
        uint4 v;
        if (src) {
            v = *reinterpret_cast<const uint4*>(src + (size_t)row * 128 + chunk * 16);
        } else {
            const uint32_t w = pattern * 0x01010101u;
            v = make_uint4(w, w, w, w);
        }
        *reinterpret_cast<uint4*>(dst + sw128_offset(row, chunk * 16)) = v;
    }
}

__global__ void __launch_bounds__(kThreads, 1) pv_kernel(const Params p) {
    extern __shared__ uint8_t smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t warp = warp_id_uniform();
    const uint32_t lane = lane_id();
    const int slot_off = (int)(blockIdx.x % kSlotStride);

    if (threadIdx.x == 0) {
        for (int r = 0; r < GPLK_PV_ROLE_COUNT; ++r) sm.role_count[r] = 0;
        for (int w = 0; w < kWarps; ++w) {
            const int r = p.role_map[(w * kSlotStride + slot_off) % GPLK_PV_ROLE_SLOTS] & 7;
            sm.role_of[w] = (unsigned char)r;
            sm.role_rank[w] = sm.role_count[r]++;
        }
        for (int s = 0; s < kRingStages; ++s) mbar_init(&sm.ring_full[s], 1);
        mbar_init(&sm.mma_done, 1);
        sm.has_tmem = 0;
        sm.abort = 0;
        fence_barrier_init();
    }
    __syncthreads();

    const int role = sm.role_of[warp];
    const int rank = sm.role_rank[warp];
    const int inner = p.inner;
    // Time-boxed mode: after its fixed `inner` work, every role keeps going in
    // small rounds until the shared deadline, so all units stay busy for the
    // whole launch instead of the fastest roles idling behind the slowest.
    const uint64_t deadline = p.budget_ns ? globaltimer_ns() + p.budget_ns : 0;
    auto more = [&]() -> bool { return deadline != 0 && globaltimer_ns() < deadline && !*(volatile int*)&sm.abort; };
    const uint32_t global_warp = blockIdx.x * kWarps + warp;
    uint32_t keep_bits = 0;
    float keep = 0.0f;

    if (role == GPLK_PV_ROLE_TENSOR) {
        if (rank == 0) {
            fill_tile(sm.mma_a, p.mma_a, 128, 0x38, lane);  // 0x38 = E4M3 1.0
            fill_tile(sm.mma_b, p.mma_b, 256, 0x38, lane);
            fence_proxy_async_smem();  // generic writes -> visible to the tensor core
            __syncwarp();
            tmem_alloc(&sm.tmem_base, kTmemCols);
            tmem_relinquish();
            tc_fence_before();
            __syncwarp();
            tc_fence_after();
            if (lane == 0) {
                sm.has_tmem = 1;
                const uint32_t d = sm.tmem_base;
                const uint32_t a0 = smem_u32(sm.mma_a), b0 = smem_u32(sm.mma_b);
                const uint32_t idesc = idesc_e4m3_f32(128, 256);
                int tiles = inner;
                for (int it = 0;; ++it) {
                    if (it == tiles) {
                        if (!more()) break;
                        tiles += 16;
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        mma_f8f6f4(d, desc_kmajor_sw128(a0 + 32 * j), desc_kmajor_sw128(b0 + 32 * j), idesc,
                                   (it | j) != 0);
                    if ((it & 255) == 255 && *(volatile int*)&sm.abort) break;
                }
                tc_commit(&sm.mma_done);
                int dummy = 0;
                mbar_wait(&sm.mma_done, 0, &dummy, 0x0301);
            }
            __syncwarp();
        }
        // Other tensor-role warps have no instruction to issue: they park.
    } else if (role == GPLK_PV_ROLE_FMA) {
        float x0 = 1.0001f + (float)lane, x1 = 1.0002f, x2 = 1.0003f, x3 = 1.0004f;
        float x4 = 1.0005f, x5 = 1.0006f, x6 = 1.0007f, x7 = 1.0008f;
        const float m = 0.9999f, c = 1e-7f;
        for (int steps = inner * 16;; steps = 256) {
            for (int i = 0; i < steps; ++i) {
                x0 = __fmaf_rn(x0, m, c); x1 = __fmaf_rn(x1, m, c);
                x2 = __fmaf_rn(x2, m, c); x3 = __fmaf_rn(x3, m, c);
                x4 = __fmaf_rn(x4, m, c); x5 = __fmaf_rn(x5, m, c);
                x6 = __fmaf_rn(x6, m, c); x7 = __fmaf_rn(x7, m, c);
            }
            if (!more()) break;
        }
        keep = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(x0, x1), x2), x3), x4), x5), x6), x7);
        keep_bits = __float_as_uint(keep);
    } else if (role == GPLK_PV_ROLE_DRAM && rank >= kRingStages) {
        // More DRAM warps than ring stages: the extra warps stream with
        // L2-missing strided 128-bit loads, as the reference's DRAM role does.
        const size_t stride = 65537;
        size_t idx = ((size_t)global_warp * 2654435761u + lane) % p.stream_elems;
        float acc = 0.0f;
        for (int loads = inner * 4;; loads = 64) {
            for (int i = 0; i < loads; ++i) {
                const float4 v = p.stream_buf[idx];
                acc += v.x + v.y + v.z + v.w;
                idx += stride;
                if (idx >= p.stream_elems) idx -= p.stream_elems;
            }
            if (!more()) break;
        }
        keep = acc;
        keep_bits = __float_as_uint(acc);
    } else if (role == GPLK_PV_ROLE_DRAM) {
        if (lane == 0 && p.stream_chunks > 0) {
            const int nd = min(sm.role_count[GPLK_PV_ROLE_DRAM], kRingStages);
            // This warp's stages: rank, rank + nd, ... (at least one, as rank < 16).
            int mine[kRingStages];
            int n_mine = 0;
            for (int s = rank; s < kRingStages; s += nd) mine[n_mine++] = s;
            const long long chunks = inner > 4 ? inner / 4 : 1;
            const size_t G = (size_t)gridDim.x * kWarps;
            const char* src = reinterpret_cast<const char*>(p.stream_buf);
            long long j = 0;
            bool ok = true;
            for (long long limit = chunks; j < limit || (more() && (limit = j + 1)); ++j) {
                const int st = mine[j % n_mine];
                if (j >= n_mine) {
                    const uint32_t par = (uint32_t)(((j / n_mine) - 1) & 1);
                    if (!mbar_wait(&sm.ring_full[st], par, &sm.abort, 0x0311)) { ok = false; break; }
                }
                const size_t chunk = ((size_t)global_warp + (size_t)j * G) % p.stream_chunks;
                mbar_arrive_expect_tx(&sm.ring_full[st], kChunk);
                bulk_load(sm.ring[st], src + chunk * kChunk, kChunk, &sm.ring_full[st]);
            }
            // Drain: the last load of each owned stage lands before exit.
            int dummy = 0;
            const long long issued = j;
            for (int q = 0; q < n_mine && q < issued; ++q) {
                const long long last = issued - 1 - ((issued - 1 - q) % n_mine);
                const uint32_t par = (uint32_t)((last / n_mine) & 1);
                mbar_wait(&sm.ring_full[mine[last % n_mine]], par, &dummy, 0x0312, 100000000ull);
            }
            keep_bits = ok ? 0u : 1u;
        }
    } else if (role == GPLK_PV_ROLE_L2) {
        // The window never exceeds the buffer, so every read stays in bounds
        // for the smallest buffer the launcher accepts (64 KiB).
        const size_t win = min(kL2WindowBytes / sizeof(float4), p.stream_elems);
        const size_t base = ((size_t)blockIdx.x * 977) % (p.stream_elems > win ? p.stream_elems - win : 1);
        size_t idx = lane;
        float acc = 0.0f;
        for (int loads = inner * 4;; loads = 64) {
            for (int i = 0; i < loads; ++i) {
                const float4 v = p.stream_buf[base + (idx % win)];
                acc += v.x + v.y + v.z + v.w;
                idx += 129;
            }
            if (!more()) break;
        }
        keep = acc;
        keep_bits = __float_as_uint(acc);
    } else if (role == GPLK_PV_ROLE_SFU) {
        float a0 = 0.7f + lane * 0.01f, a1 = 1.1f, a2 = 0.3f, a3 = 1.7f;
        for (int steps = inner * 4;; steps = 64) {
            for (int i = 0; i < steps; ++i) {
                a0 = __sinf(a0) + 1.0f;
                a1 = __expf(a1 * 0.5f) * 0.5f;
                a2 = __logf(a2 + 2.0f);
                a3 = __frsqrt_rn(a3 + 1.0f) + 1.0f;
            }
            if (!more()) break;
        }
        keep = a0 + a1 + a2 + a3;
        keep_bits = __float_as_uint(keep);
    } else if (role == GPLK_PV_ROLE_INT32) {
        uint32_t i0 = 0x9E3779B9u + lane, i1 = 0x85EBCA6Bu, i2 = 0xC2B2AE35u, i3 = 0x27D4EB2Fu;
        for (int steps = inner * 16;; steps = 256) {
            for (int i = 0; i < steps; ++i) {
                i0 = i0 * 1664525u + 1013904223u;
                i1 = i1 * 22695477u + 1u;
                i2 = i2 * 1103515245u + 12345u;
                i3 = i3 * 214013u + 2531011u;
            }
            if (!more()) break;
        }
        keep_bits = i0 ^ i1 ^ i2 ^ i3;
        keep = (float)(keep_bits & 0xFFFFu);
    } else if (role == GPLK_PV_ROLE_SMEM) {
        float* mine = sm.smem_role[warp];
        mine[lane] = 1.0f + lane;
        mine[lane + 32] = 2.0f;
        __syncwarp();
        float acc = 0.0f;
        int i = 0;
        for (int steps = inner * 8;; steps = 256) {
            for (const int end = i + steps; i < end; ++i) {
                const int j = (lane + i) & 31;
                acc = __fmaf_rn(mine[j], 1.000001f, acc);
                mine[j + 32] = acc;
            }
            if (!more()) break;
        }
        keep = acc;
        keep_bits = __float_as_uint(acc);
    } else {  // ATOMIC
        float acc = 0.0f;
        const int slot = (int)((global_warp * 32 + lane) & (kAtomicSlots - 1));
        for (int ops = inner;; ops = 16) {
            for (int i = 0; i < ops; ++i) acc += atomicAdd(&p.sink[1 + slot], 1.0f);
            if (!more()) break;
        }
        keep = acc * 1e-30f;
        keep_bits = __float_as_uint(keep);
    }

    if (keep == 1.2345678e-30f) p.sink[0] = keep;  // never true; keeps the work live
    if (p.verify_out) p.verify_out[(size_t)global_warp * 32 + lane] = keep_bits;

    __syncwarp();  // roles leave lanes diverged: reconverge before the block-wide barrier
    tc_fence_before();
    __syncthreads();
    if (sm.has_tmem) {
        if (p.mma_out && blockIdx.x == 0 && warp < 4) {
            tc_fence_after();
            const uint32_t taddr = sm.tmem_base + ((warp * 32u) << 16);
            const uint32_t row = warp * 32 + lane;
            // 16 columns per load: the kernel's 64-register budget (1024 threads) holds no more
            for (int c = 0; c < 16; ++c) {
                uint32_t r[16];
                tmem_ld_32x32b_x16(taddr + 16u * c, r);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) p.mma_out[(size_t)row * 256 + c * 16 + j] = __uint_as_float(r[j]);
            }
        }
        __syncwarp();
        tc_fence_before();
        __syncthreads();
        if (role == GPLK_PV_ROLE_TENSOR && rank == 0) {
            tc_fence_after();
            tmem_dealloc(sm.tmem_base, kTmemCols);
        }
    }
}

}  // namespace pv
}  // namespace gplk

extern "C" int gplk_pv_block_threads(void) { return gplk::pv::kThreads; }

extern "C" void gplk_pv_build_role_map(const int weights[GPLK_PV_ROLE_COUNT], unsigned char* map,
                                       int* counts) {
    // Largest-remainder apportionment (runner/src/workload_powervirus.cu:414-454):
    // floor shares, a non-zero weight never rounds to zero, excess trimmed
    // from the largest share, the rest handed out by largest remainder.
    constexpr int R = GPLK_PV_ROLE_COUNT, S = GPLK_PV_ROLE_SLOTS;
    int w[R], share[R];
    double frac[R];
    long total = 0;
    for (int r = 0; r < R; ++r) {
        w[r] = weights[r] > 0 ? weights[r] : 0;
        total += w[r];
    }
    if (total == 0) {
        w[GPLK_PV_ROLE_FMA] = 1;
        total = 1;
    }
    int given = 0;
    for (int r = 0; r < R; ++r) {
        const double exact = (double)S * w[r] / (double)total;
        share[r] = (int)exact;
        frac[r] = exact - share[r];
        if (w[r] > 0 && share[r] == 0) share[r] = 1;
        given += share[r];
    }
    while (given > S) {
        int big = 0;
        for (int r = 1; r < R; ++r)
            if (share[r] > share[big]) big = r;
        --share[big];
        --given;
    }
    while (given < S) {
        int pick = -1;
        double best = -1.0;
        for (int r = 0; r < R; ++r)
            if (w[r] > 0 && frac[r] > best) {
                best = frac[r];
                pick = r;
            }
        if (pick < 0) pick = GPLK_PV_ROLE_FMA;
        ++share[pick];
        frac[pick] = -1.0;
        ++given;
    }
    int i = 0;
    for (int r = 0; r < R; ++r) {
        if (counts) counts[r] = share[r];
        for (int k = 0; k < share[r] && i < S; ++k) map[i++] = (unsigned char)r;
    }
    while (i < S) map[i++] = GPLK_PV_ROLE_FMA;
}

extern "C" int gplk_powervirus_launch(const gplk_pv_cfg* cfg, cudaStream_t stream) {
    using namespace gplk;
    if (!cfg || !cfg->role_map || !cfg->sink || cfg->inner <= 0 || cfg->blocks < 0) return GPLK_STATUS_BAD_ARG;
    if (!cfg->stream_buf || cfg->stream_bytes < (64u << 10) || (cfg->stream_bytes & 15u)) return GPLK_STATUS_BAD_ARG;
    if (!aligned16(cfg->stream_buf)) return GPLK_STATUS_BAD_ARG;
    if ((cfg->mma_a && !aligned16(cfg->mma_a)) || (cfg->mma_b && !aligned16(cfg->mma_b))) return GPLK_STATUS_BAD_ARG;
    DeviceInfo d;
    int st = require_sm100(&d);
    if (st != GPLK_STATUS_OK) return st;
    const int smem = (int)sizeof(pv::Smem) + 1024;
    if (smem > d.max_smem_optin) return GPLK_STATUS_UNSUPPORTED;
    static thread_local uint64_t configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured & (1ull << dev))) {
        if (cudaFuncSetAttribute(pv::pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return GPLK_STATUS_LAUNCH_FAIL;
        configured |= 1ull << dev;
    }
    pv::Params p;
    p.role_map = cfg->role_map;
    p.stream_buf = reinterpret_cast<const float4*>(cfg->stream_buf);
    p.stream_elems = cfg->stream_bytes / sizeof(float4);
    p.stream_chunks = cfg->stream_bytes / pv::kChunk;
    p.sink = cfg->sink;
    p.verify_out = reinterpret_cast<uint32_t*>(cfg->verify_out);
    p.mma_a = cfg->mma_a;
    p.mma_b = cfg->mma_b;
    p.mma_out = cfg->mma_out;
    p.inner = cfg->inner;
    p.budget_ns = cfg->budget_ns;
    const int grid = cfg->blocks > 0 ? cfg->blocks : d.sm_count;
    pv::pv_kernel<<<grid, pv::kThreads, smem, stream>>>(p);
    return launch_status(cudaGetLastError());
}
