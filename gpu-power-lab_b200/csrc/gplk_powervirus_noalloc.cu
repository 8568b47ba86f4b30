// gplk_powervirus_noalloc.cu - the powervirus launch for callers that cannot
// allocate device memory.
//
// gplk_powervirus_launch works on two buffers whose contents nobody reads:
// the streaming buffer behind the DRAM and L2 roles, and the atomic sink.
// Its caller has to cudaMalloc them. Some callers cannot:
//   - a load generator injected into another application's process, where
//     that application's allocator (a framework's caching allocator, an MPS
//     client limit) owns and budgets the device memory, so an extra
//     cudaMalloc fails or takes memory the application counts on;
//   - a duty-cycled burst loop, where cudaMalloc/cudaFree may synchronise the
//     device and would cut an idle gap into the power wave being measured.
// This entry point keeps both buffers in one file-scope device array instead,
// sized for at most GPLK_PV_NOALLOC_MAX_STREAM_BYTES of streaming window plus
// the sink. Every GPU that loads libgplk holds the array until the process
// exits.
//
// Every call, with the caller's device current, looks up the array's device
// address on that device with cudaGetSymbolAddress (the array's name in host
// code is only a host-side stand-in, never a device address), then, ordered
// on the caller's stream, fills the requested streaming window with a byte
// pattern and clears the sink (the atomics of the previous call leave their
// counts in it) before the launch. Nothing is cached between calls, so a
// call never uses an address or contents left from before a cudaDeviceReset,
// and no call synchronises. All calls share the array: calls that overlap on
// the GPU (other streams, other threads) race on the window and the sink.
#include <cstdio>

#include "gplk_ptx.cuh"

namespace gplk {
namespace pv_noalloc {

constexpr size_t kSinkBytes = 8192;  // 1 + 1024 floats, rounded up to 256-byte granules
constexpr size_t kMaxStreamBytes = GPLK_PV_NOALLOC_MAX_STREAM_BYTES;
constexpr size_t kScratchBytes = kSinkBytes + kMaxStreamBytes;
constexpr unsigned char kStreamPattern = 0x3c;

static __device__ __align__(256) unsigned char g_pv_scratch[kScratchBytes];

// The array's device address on the current device.
static int device_scratch(unsigned char** base) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_pv_scratch) != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        return GPLK_STATUS_CUDA_ERROR;
    }
    *base = static_cast<unsigned char*>(p);
    return GPLK_STATUS_OK;
}

}  // namespace pv_noalloc
}  // namespace gplk

extern "C" int gplk_powervirus_launch_noalloc(const unsigned char* role_map, size_t stream_bytes, int blocks,
                                              int inner, float* verify_out, const uint8_t* mma_a,
                                              const uint8_t* mma_b, float* mma_out, cudaStream_t stream) {
    using namespace gplk;
    namespace nz = gplk::pv_noalloc;
    if (!role_map || inner <= 0 || blocks < 0) return GPLK_STATUS_BAD_ARG;
    if (stream_bytes > nz::kMaxStreamBytes) {
        fprintf(stderr,
                "gplk_powervirus_launch_noalloc: stream_bytes %zu exceeds the static scratch maximum of "
                "%zu bytes (GPLK_PV_NOALLOC_MAX_STREAM_BYTES); use gplk_powervirus_launch with a caller "
                "buffer for larger windows\n",
                stream_bytes, (size_t)nz::kMaxStreamBytes);
        return GPLK_STATUS_BAD_ARG;
    }
    if (stream_bytes < (64u << 10) || (stream_bytes & 15u)) return GPLK_STATUS_BAD_ARG;
    if ((mma_a && !aligned16(mma_a)) || (mma_b && !aligned16(mma_b))) return GPLK_STATUS_BAD_ARG;
    DeviceInfo d;
    int st = require_sm100(&d);
    if (st != GPLK_STATUS_OK) return st;
    const int smem = (int)sizeof(pv::Smem) + 1024;
    if (smem > d.max_smem_optin) return GPLK_STATUS_UNSUPPORTED;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GPLK_STATUS_CUDA_ERROR;
    unsigned char* base = nullptr;
    st = nz::device_scratch(&base);
    if (st != GPLK_STATUS_OK) return st;
    static thread_local uint64_t configured = 0;
    if (!(configured & (1ull << dev))) {
        if (cudaFuncSetAttribute(pv::pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return GPLK_STATUS_LAUNCH_FAIL;
        configured |= 1ull << dev;
    }
    // The window holds the pattern a caller's buffer would be filled with, and
    // the sink starts at zero, as a freshly cleared caller sink would.
    if (cudaMemsetAsync(base + nz::kSinkBytes, nz::kStreamPattern, stream_bytes, stream) != cudaSuccess ||
        cudaMemsetAsync(base, 0, nz::kSinkBytes, stream) != cudaSuccess)
        return GPLK_STATUS_CUDA_ERROR;
    pv::Params p;
    p.role_map = role_map;
    p.stream_buf = reinterpret_cast<const float4*>(base + nz::kSinkBytes);
    p.stream_elems = stream_bytes / sizeof(float4);
    p.stream_chunks = stream_bytes / pv::kChunk;
    p.sink = reinterpret_cast<float*>(base);
    p.verify_out = reinterpret_cast<uint32_t*>(verify_out);
    p.mma_a = mma_a;
    p.mma_b = mma_b;
    p.mma_out = mma_out;
    p.inner = inner;
    p.budget_ns = 0;  // fixed work, as gplk_powervirus_launch with budget_ns = 0
    const int grid = blocks > 0 ? blocks : d.sm_count;
    pv::pv_kernel<<<grid, pv::kThreads, smem, stream>>>(p);
    return launch_status(cudaGetLastError());
}
