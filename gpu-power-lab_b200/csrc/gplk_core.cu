// gplk_core.cu - status word, device checks and TMA descriptor encoding
// shared by every launcher in libgplk. Compiled as part of gplk_unity.cu.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <utility>

#include "gplk_ptx.cuh"

namespace gplk {

// Per-device facts needed at launch time, looked up once per device.
struct DeviceInfo {
    int sm_count = 0;
    int major = 0;
    int minor = 0;
    int max_smem_optin = 0;
    bool valid = false;
};

static DeviceInfo g_devinfo[64];
static std::mutex g_devinfo_mu;

static int current_device_info(DeviceInfo* out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GPLK_STATUS_CUDA_ERROR;
    std::lock_guard<std::mutex> lock(g_devinfo_mu);
    DeviceInfo& d = g_devinfo[dev];
    if (!d.valid) {
        if (cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
                cudaSuccess) {
            return GPLK_STATUS_CUDA_ERROR;
        }
        d.valid = true;
    }
    *out = d;
    return GPLK_STATUS_OK;
}

// The tcgen05 kernels are built for sm_100a only; refuse anything else
// instead of failing inside the launch.
static int require_sm100(DeviceInfo* info) {
    int st = current_device_info(info);
    if (st != GPLK_STATUS_OK) return st;
    if (info->major != 10 || info->minor != 0) return GPLK_STATUS_UNSUPPORTED;
    return GPLK_STATUS_OK;
}

static int launch_status(cudaError_t e) {
    if (e == cudaSuccess) return GPLK_STATUS_OK;
    return GPLK_STATUS_LAUNCH_FAIL;
}

// Launches `kernel` with programmatic stream serialisation, so it may begin
// (up to its pdl_wait()) while the previous kernel on `stream` finishes.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// cuTensorMapEncodeTiled reached through the runtime's driver entry point,
// so the library does not link libcuda directly.
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        }
    });
    return fn;
}

// 2-D byte tensor: `rows` rows of `row_bytes` bytes, row pitch `pitch`.
// Box of box_rows x box_bytes with 128-byte swizzle (box_bytes <= 128).
// Out-of-range elements of a box are filled with zeros by the TMA unit.
static int encode_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows,
                             uint64_t pitch, uint32_t box_bytes, uint32_t box_rows,
                             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    auto enc = tensor_map_encoder();
    if (!enc) return GPLK_STATUS_UNSUPPORTED;
    cuuint64_t dims[2] = {row_bytes, rows};
    cuuint64_t strides[1] = {pitch};
    cuuint32_t box[2] = {box_bytes, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? GPLK_STATUS_OK : GPLK_STATUS_BAD_ARG;
}

// 2-D 16-bit tensor, row length `inner` elements, `outer` rows, row pitch
// `pitch_bytes`; box inner x outer, no swizzle (for TMA stores of BF16 tiles).
static int encode_tmap_2d_u16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                              uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
    auto enc = tensor_map_encoder();
    if (!enc) return GPLK_STATUS_UNSUPPORTED;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {pitch_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? GPLK_STATUS_OK : GPLK_STATUS_BAD_ARG;
}

// The same for 32-bit elements (TMA stores of FP32 / S32 tiles).
static int encode_tmap_2d_u32(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                              uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer) {
    auto enc = tensor_map_encoder();
    if (!enc) return GPLK_STATUS_UNSUPPORTED;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {pitch_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? GPLK_STATUS_OK : GPLK_STATUS_BAD_ARG;
}

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace gplk

extern "C" const char* gplk_status_string(int status) {
    switch (status) {
        case GPLK_STATUS_OK: return "ok";
        case GPLK_STATUS_BAD_ARG: return "bad argument";
        case GPLK_STATUS_LAUNCH_FAIL: return "kernel launch failed";
        case GPLK_STATUS_DEVICE_TIMEOUT: return "device wait timeout";
        case GPLK_STATUS_UNSUPPORTED: return "unsupported device";
        case GPLK_STATUS_CUDA_ERROR: return "cuda error";
        default: return "unknown status";
    }
}

extern "C" int gplk_abi_version(void) { return 3; }

extern "C" int gplk_status_read(int* code, int* site, int clear) {
    if (cudaDeviceSynchronize() != cudaSuccess) return GPLK_STATUS_CUDA_ERROR;
    int c = 0, s = 0;
    if (cudaMemcpyFromSymbol(&c, gplk::g_status, sizeof(int)) != cudaSuccess) return GPLK_STATUS_CUDA_ERROR;
    if (cudaMemcpyFromSymbol(&s, gplk::g_status_site, sizeof(int)) != cudaSuccess)
        return GPLK_STATUS_CUDA_ERROR;
    if (code) *code = c;
    if (site) *site = s;
    if (clear) {
        int zero = 0;
        if (cudaMemcpyToSymbol(gplk::g_status, &zero, sizeof(int)) != cudaSuccess ||
            cudaMemcpyToSymbol(gplk::g_status_site, &zero, sizeof(int)) != cudaSuccess)
            return GPLK_STATUS_CUDA_ERROR;
    }
    return GPLK_STATUS_OK;
}

// ------------------------------------------------------------ watchdog self-test
namespace gplk {
// One block waits on an mbarrier that nothing ever arrives on. The bounded
// wait must give up after budget_ns, record GPLK_STATUS_DEVICE_TIMEOUT with
// site 0x0F01 and let the block exit normally.
__global__ void selftest_wait_kernel(uint64_t budget_ns, int* gave_up) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const bool ok = mbar_wait(&bar, 0, &abort_flag, 0x0F01, budget_ns);
    if (threadIdx.x == 0 && gave_up) *gave_up = ok ? 0 : 1;
}
}  // namespace gplk

extern "C" int gplk_selftest_wait_timeout(unsigned long long budget_ns, int* gave_up, cudaStream_t stream) {
    if (budget_ns == 0 || budget_ns > 2000000000ull) return GPLK_STATUS_BAD_ARG;
    gplk::selftest_wait_kernel<<<1, 32, 0, stream>>>(budget_ns, gave_up);
    return gplk::launch_status(cudaGetLastError());
}
