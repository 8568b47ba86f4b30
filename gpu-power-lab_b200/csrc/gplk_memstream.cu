// gplk_memstream.cu - STREAM triad and copy for B200 HBM3e.
//
// Two triad kernels, both bit-exact against a host fmaf loop:
//   triad_vec4  - 128-bit LDG/STG grid-stride loop over a persistent grid of
//                 (SMs x resident blocks); each thread keeps UNROLL float4
//                 loads of each operand in flight. Streaming cache hints:
//                 operands are touched once, so they should not displace
//                 anything from L2.
//   triad_bulk  - operands staged through shared memory by 1-D TMA bulk
//                 copies (cp.async.bulk) in a STAGES-deep ring, results
//                 written back with bulk stores from shared memory.
// Algorithmic traffic is 12 bytes per element (read b, read c, write a),
// the accounting of runner/src/workload_util.c:43-47.
#include "gplk_ptx.cuh"

namespace gplk {
namespace memstream {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }

__device__ __forceinline__ float4 triad4(float s, float4 b, float4 c) {
    float4 r;
    r.x = __fmaf_rn(s, c.x, b.x);
    r.y = __fmaf_rn(s, c.y, b.y);
    r.z = __fmaf_rn(s, c.z, b.z);
    r.w = __fmaf_rn(s, c.w, b.w);
    return r;
}

// n4 = number of float4 elements; tail = n % 4 scalar elements after them.
__global__ void __launch_bounds__(kThreads) triad_vec4(float4* __restrict__ a,
                                                       const float4* __restrict__ b,
                                                       const float4* __restrict__ c, float s,
                                                       size_t n4, int tail) {
    const size_t stride = (size_t)gridDim.x * kThreads;
    size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x;
    // Main body: kUnroll independent float4 pairs in flight per thread.
    for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
        float4 bv[kUnroll], cv[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            bv[u] = ld_stream(b + i + u * stride);
            cv[u] = ld_stream(c + i + u * stride);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) st_stream(a + i + u * stride, triad4(s, bv[u], cv[u]));
    }
    for (; i < n4; i += stride) st_stream(a + i, triad4(s, ld_stream(b + i), ld_stream(c + i)));
    if (tail && blockIdx.x == 0 && threadIdx.x < tail) {
        const float* bs = reinterpret_cast<const float*>(b + n4);
        const float* cs = reinterpret_cast<const float*>(c + n4);
        float* as = reinterpret_cast<float*>(a + n4);
        as[threadIdx.x] = __fmaf_rn(s, cs[threadIdx.x], bs[threadIdx.x]);
    }
}

// Fallback for operands that are not 16-byte aligned.
__global__ void __launch_bounds__(kThreads) triad_scalar(float* __restrict__ a,
                                                         const float* __restrict__ b,
                                                         const float* __restrict__ c, float s,
                                                         size_t n) {
    const size_t stride = (size_t)gridDim.x * kThreads;
    for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride)
        a[i] = __fmaf_rn(s, __ldcs(c + i), __ldcs(b + i));
}

__global__ void __launch_bounds__(kThreads) copy_vec4(float4* __restrict__ dst,
                                                      const float4* __restrict__ src, size_t n4,
                                                      int tail) {
    const size_t stride = (size_t)gridDim.x * kThreads;
    size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x;
    for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
        float4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = ld_stream(src + i + u * stride);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) st_stream(dst + i + u * stride, v[u]);
    }
    for (; i < n4; i += stride) st_stream(dst + i, ld_stream(src + i));
    if (tail && blockIdx.x == 0 && threadIdx.x < tail) {
        reinterpret_cast<float*>(dst + n4)[threadIdx.x] =
            reinterpret_cast<const float*>(src + n4)[threadIdx.x];
    }
}

__global__ void __launch_bounds__(kThreads) copy_scalar(float* __restrict__ dst,
                                                        const float* __restrict__ src, size_t n) {
    const size_t stride = (size_t)gridDim.x * kThreads;
    for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += stride)
        dst[i] = __ldcs(src + i);
}

// ------------------------------------------------------------ TMA bulk triad

constexpr int kBulkThreads = 256;
constexpr int kBulkChunk = 4096;  // floats per operand per stage (16 KiB)
constexpr int kBulkStages = 4;    // 4 x 2 x 16 KiB = 128 KiB of ring

struct BulkSmem {
    float b[kBulkStages][kBulkChunk];
    float c[kBulkStages][kBulkChunk];
    uint64_t full[kBulkStages];
    int abort;
};

// Chunks are distributed round-robin over a persistent grid. Thread 0 issues
// every bulk copy; all threads compute. The result overwrites the b buffer in
// shared memory and is stored from there. Elements past the last whole
// float4 are handled by the caller's scalar tail launch.
__global__ void __launch_bounds__(kBulkThreads) triad_bulk(float* __restrict__ a,
                                                           const float* __restrict__ b,
                                                           const float* __restrict__ c, float s,
                                                           size_t n_vec /* multiple of 4 */) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    BulkSmem& sm = *reinterpret_cast<BulkSmem*>(smem_raw);
    const size_t nchunks = (n_vec + kBulkChunk - 1) / kBulkChunk;
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < kBulkStages; ++i) mbar_init(&sm.full[i], 1);
        sm.abort = 0;
        fence_barrier_init();
    }
    __syncthreads();

    // Local index j -> global chunk blockIdx.x + j * gridDim.x.
    const size_t my_chunks =
        (blockIdx.x < nchunks) ? (nchunks - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;

    auto chunk_elems = [&](size_t chunk) -> uint32_t {
        size_t first = chunk * kBulkChunk;
        size_t left = n_vec - first;
        return (uint32_t)(left < (size_t)kBulkChunk ? left : (size_t)kBulkChunk);
    };
    auto issue = [&](size_t j) {
        const int st = (int)(j % kBulkStages);
        const size_t chunk = blockIdx.x + j * gridDim.x;
        const uint32_t bytes = chunk_elems(chunk) * 4u;
        mbar_arrive_expect_tx(&sm.full[st], 2u * bytes);
        bulk_load(sm.b[st], b + chunk * kBulkChunk, bytes, &sm.full[st]);
        bulk_load(sm.c[st], c + chunk * kBulkChunk, bytes, &sm.full[st]);
    };

    if (tid == 0) {
        for (size_t j = 0; j < my_chunks && j < (size_t)kBulkStages - 1; ++j) issue(j);
    }
    size_t completed = 0;  // chunks whose loads were waited on (for drain)
    for (size_t j = 0; j < my_chunks; ++j) {
        const int st = (int)(j % kBulkStages);
        if (tid == 0 && j + kBulkStages - 1 < my_chunks) {
            // The stage about to be refilled was last stored from at j - 1;
            // wait until that store has finished reading shared memory.
            bulk_wait_read<0>();
            issue(j + kBulkStages - 1);
        }
        const uint32_t parity = (uint32_t)((j / kBulkStages) & 1);
        const bool ok = mbar_wait(&sm.full[st], parity, &sm.abort, 0x0101);
        if (__syncthreads_or(!ok)) break;  // every thread leaves together
        completed = j + 1;
        const size_t chunk = blockIdx.x + j * gridDim.x;
        const uint32_t elems = chunk_elems(chunk);
        float4* bb = reinterpret_cast<float4*>(sm.b[st]);
        const float4* cc = reinterpret_cast<const float4*>(sm.c[st]);
        for (uint32_t v = tid; v < elems / 4; v += kBulkThreads) bb[v] = triad4(s, bb[v], cc[v]);
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the bulk store
        __syncthreads();
        if (tid == 0) {
            bulk_store(a + chunk * kBulkChunk, sm.b[st], elems * 4u);
            bulk_commit();
        }
    }
    if (tid == 0) {
        if (sm.abort) {
            // Let every load this thread issued land before the block exits.
            size_t issued = my_chunks < completed + kBulkStages ? my_chunks : completed + kBulkStages;
            int dummy = 0;
            for (size_t j = completed; j < issued; ++j) {
                mbar_wait(&sm.full[j % kBulkStages], (uint32_t)((j / kBulkStages) & 1), &dummy,
                          0x0102, 100000000ull);
            }
        }
        bulk_wait<0>();
    }
    __syncthreads();
}

static int grid_for(const DeviceInfo& d, size_t work_items, int per_sm) {
    size_t want = (work_items + kThreads - 1) / kThreads;
    size_t cap = (size_t)d.sm_count * per_sm;
    if (want > cap) want = cap;
    if (want < 1) want = 1;
    return (int)want;
}

}  // namespace memstream
}  // namespace gplk

using namespace gplk;

extern "C" int gplk_triad_f32(float* a, const float* b, const float* c, float s, size_t n,
                              cudaStream_t stream) {
    if (n == 0) return GPLK_STATUS_OK;
    if (!a || !b || !c) return GPLK_STATUS_BAD_ARG;
    DeviceInfo d;
    int st = current_device_info(&d);
    if (st != GPLK_STATUS_OK) return st;
    if (aligned16(a) && aligned16(b) && aligned16(c)) {
        size_t n4 = n / 4;
        int tail = (int)(n % 4);
        int grid = memstream::grid_for(d, n4 ? n4 : 1, 8);
        memstream::triad_vec4<<<grid, memstream::kThreads, 0, stream>>>(
            reinterpret_cast<float4*>(a), reinterpret_cast<const float4*>(b),
            reinterpret_cast<const float4*>(c), s, n4, tail);
    } else {
        int grid = memstream::grid_for(d, n, 8);
        memstream::triad_scalar<<<grid, memstream::kThreads, 0, stream>>>(a, b, c, s, n);
    }
    return launch_status(cudaGetLastError());
}

extern "C" int gplk_copy_f32(float* dst, const float* src, size_t n, cudaStream_t stream) {
    if (n == 0) return GPLK_STATUS_OK;
    if (!dst || !src) return GPLK_STATUS_BAD_ARG;
    DeviceInfo d;
    int st = current_device_info(&d);
    if (st != GPLK_STATUS_OK) return st;
    if (aligned16(dst) && aligned16(src)) {
        size_t n4 = n / 4;
        int grid = memstream::grid_for(d, n4 ? n4 : 1, 8);
        memstream::copy_vec4<<<grid, memstream::kThreads, 0, stream>>>(
            reinterpret_cast<float4*>(dst), reinterpret_cast<const float4*>(src), n4, (int)(n % 4));
    } else {
        int grid = memstream::grid_for(d, n, 8);
        memstream::copy_scalar<<<grid, memstream::kThreads, 0, stream>>>(dst, src, n);
    }
    return launch_status(cudaGetLastError());
}

extern "C" int gplk_triad_f32_bulk(float* a, const float* b, const float* c, float s, size_t n,
                                   cudaStream_t stream) {
    if (n == 0) return GPLK_STATUS_OK;
    if (!a || !b || !c) return GPLK_STATUS_BAD_ARG;
    if (!aligned16(a) || !aligned16(b) || !aligned16(c)) return GPLK_STATUS_BAD_ARG;
    DeviceInfo d;
    int st = require_sm100(&d);
    if (st != GPLK_STATUS_OK) return st;
    const size_t n_vec = n & ~(size_t)3;
    const int smem = (int)sizeof(memstream::BulkSmem);
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        if (cudaFuncSetAttribute(memstream::triad_bulk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem) != cudaSuccess)
            return GPLK_STATUS_LAUNCH_FAIL;
        configured_dev = dev;
    }
    if (n_vec) {
        size_t nchunks = (n_vec + memstream::kBulkChunk - 1) / memstream::kBulkChunk;
        size_t grid = (size_t)d.sm_count;  // 128 KiB ring -> one block per SM
        if (grid > nchunks) grid = nchunks;
        memstream::triad_bulk<<<(unsigned)grid, memstream::kBulkThreads, smem, stream>>>(a, b, c, s,
                                                                                         n_vec);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return GPLK_STATUS_LAUNCH_FAIL;
    }
    if (n != n_vec) {
        memstream::triad_scalar<<<1, memstream::kThreads, 0, stream>>>(a + n_vec, b + n_vec, c + n_vec,
                                                                       s, n - n_vec);
    }
    return launch_status(cudaGetLastError());
}
