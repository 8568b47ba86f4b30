// gplk_fabric.cu - the powervirus cycle's fabric step as one kernel over
// NVLink peer memory: an in-place BF16 sum allreduce across the GPUs of one
// node, in place of the NCCL allreduce the multi-GPU rung issues
// (runner/src/workload_nccl.cu:119-291 runs ncclAllReduce on FP32; the
// rung here reduces 256 MiB of BF16 once per duty cycle).
//
// Every rank cudaMallocs one region: a 4 KiB flag block followed by the data
// buffer. Ranks exchange CUDA IPC handles for it (the host side does the
// exchange, e.g. through torch.distributed) and map each other's regions, so
// every rank holds device pointers to all ranks' data and flags.
//
// One pass, no intermediate barrier. The buffer is cut into `world` chunks;
// rank r owns chunk r. Each thread of rank r loads one 16-byte vector of
// chunk r from every rank's buffer (peer loads over NVLink), sums the eight
// BF16 lanes in FP32 in rank order 0..world-1, rounds once to BF16, and
// stores the result into every rank's buffer at the same place (peer stores).
// This is race-free without a middle barrier: chunk r of any buffer is read
// only by rank r, and each thread reads a vector before it overwrites it.
//   entry   each rank announces the epoch to all peers and waits for all of
//           them, so every input is in place before anyone reads it;
//   exit    each rank's last block announces completion after a system-scope
//           fence; block 0 waits for all ranks, so when the kernel ends every
//           peer's stores into this rank's buffer are visible.
// Flags carry a per-fabric epoch, so nothing is ever reset. Every wait is
// bounded (2 s by default): on timeout the kernel records
// GPLK_STATUS_DEVICE_TIMEOUT with the site and returns; no trap. The grid is
// launched cooperatively (all blocks co-resident) with two blocks per SM.
// No multicast of any kind: plain peer loads and stores only.
#include <cstring>

#include "gplk_ptx.cuh"

namespace gplk {
namespace fabric {

constexpr int kMaxRanks = 8;
constexpr size_t kFlagBytes = 4096;  // flag block at the start of every region
constexpr int kEntry = 0;            // flags[kEntry + q]: rank q entered epoch
constexpr int kDone = 16;            // flags[kDone + q]: rank q finished epoch
constexpr int kCounter = 32;         // this rank's block counter (local only)
constexpr int kThreads = 512;

struct Args {
    const uint4* src[kMaxRanks];  // every rank's data buffer (16-byte vectors)
    uint4* dst[kMaxRanks];        // the same pointers, for the stores
    unsigned* flags[kMaxRanks];   // every rank's flag block
    int rank, world;
    size_t n16;       // vectors to reduce
    size_t chunk16;   // vectors per chunk (the last chunk may be shorter)
    unsigned epoch;
    unsigned long long budget_ns;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait until *flag == epoch. Returns false after recording a timeout.
__device__ __forceinline__ bool wait_flag(const unsigned* flag, unsigned epoch, unsigned long long budget_ns,
                                          int site) {
    if (ld_acquire_sys(flag) == epoch) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        __nanosleep(64);
        if (ld_acquire_sys(flag) == epoch) return true;
        if (globaltimer_ns() - t0 > budget_ns) {
            record_error(GPLK_STATUS_DEVICE_TIMEOUT, site);
            return false;
        }
    }
}

__device__ __forceinline__ void add_bf16x2(float& lo, float& hi, uint32_t v) {
    lo += __uint_as_float(v << 16);
    hi += __uint_as_float(v & 0xFFFF0000u);
}

// Sums of one 16-byte vector from every rank, in rank order 0..W-1 (so all
// ranks produce identical bits). FP32: four elements per vector.
template <int W>
__device__ __forceinline__ uint4 sum_f32(const uint4 (&v)[W]) {
    float s0 = __uint_as_float(v[0].x), s1 = __uint_as_float(v[0].y), s2 = __uint_as_float(v[0].z),
          s3 = __uint_as_float(v[0].w);
#pragma unroll
    for (int q = 1; q < W; ++q) {
        s0 += __uint_as_float(v[q].x);
        s1 += __uint_as_float(v[q].y);
        s2 += __uint_as_float(v[q].z);
        s3 += __uint_as_float(v[q].w);
    }
    return make_uint4(__float_as_uint(s0), __float_as_uint(s1), __float_as_uint(s2), __float_as_uint(s3));
}

// BF16: eight elements per vector, summed in FP32 and rounded once.
template <int W>
__device__ __forceinline__ uint4 sum_bf16(const uint4 (&v)[W]) {
    float s[8];
    s[0] = __uint_as_float(v[0].x << 16);
    s[1] = __uint_as_float(v[0].x & 0xFFFF0000u);
    s[2] = __uint_as_float(v[0].y << 16);
    s[3] = __uint_as_float(v[0].y & 0xFFFF0000u);
    s[4] = __uint_as_float(v[0].z << 16);
    s[5] = __uint_as_float(v[0].z & 0xFFFF0000u);
    s[6] = __uint_as_float(v[0].w << 16);
    s[7] = __uint_as_float(v[0].w & 0xFFFF0000u);
#pragma unroll
    for (int q = 1; q < W; ++q) {
        add_bf16x2(s[0], s[1], v[q].x);
        add_bf16x2(s[2], s[3], v[q].y);
        add_bf16x2(s[4], s[5], v[q].z);
        add_bf16x2(s[6], s[7], v[q].w);
    }
    return make_uint4(pack_bf16x2(s[0], s[1]), pack_bf16x2(s[2], s[3]), pack_bf16x2(s[4], s[5]),
                      pack_bf16x2(s[6], s[7]));
}

// Reduces U vectors, `stride` apart from index i, and pushes each sum to
// every rank. All U x W loads are in flight before the first sum.
template <int W, bool F32, int U>
__device__ __forceinline__ void reduce_push(const Args& a, size_t i, size_t stride) {
    uint4 v[U][W];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
        for (int q = 0; q < W; ++q) v[u][q] = a.src[q][i + u * stride];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const uint4 r = F32 ? sum_f32<W>(v[u]) : sum_bf16<W>(v[u]);
#pragma unroll
        for (int q = 0; q < W; ++q) a.dst[q][i + u * stride] = r;
    }
}

template <int W, bool F32>
__global__ void __launch_bounds__(kThreads, 2) allreduce_kernel(const Args a) {
    unsigned* my_flags = a.flags[a.rank];
    // ---- entry: announce, then wait for every rank (one thread per block)
    if (blockIdx.x == 0 && threadIdx.x < (unsigned)W) st_release_sys(a.flags[threadIdx.x] + kEntry + a.rank, a.epoch);
    __shared__ int ok;
    if (threadIdx.x == 0) {
        bool good = true;
        for (int q = 0; q < W && good; ++q) good = wait_flag(my_flags + kEntry + q, a.epoch, a.budget_ns, 0x0701);
        ok = good;
    }
    __syncthreads();
    if (ok) {
        // ---- reduce this rank's chunk and push the sums to every rank
        const size_t lo = (size_t)a.rank * a.chunk16;
        const size_t hi = lo + a.chunk16 < a.n16 ? lo + a.chunk16 : a.n16;
        const size_t stride = (size_t)gridDim.x * blockDim.x;
        // Two vectors per thread per step: 2 x W loads in flight. Measured
        // at N = 2, 256 MiB: 623 -> 648 GB/s bus bandwidth (655 together
        // with two blocks per SM).
        size_t i = lo + (size_t)blockIdx.x * blockDim.x + threadIdx.x;
        for (; i + stride < hi; i += 2 * stride) reduce_push<W, F32, 2>(a, i, stride);
        if (i < hi) reduce_push<W, F32, 1>(a, i, stride);
    }
    // ---- exit: the last block of this rank tells every rank, block 0 waits
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(my_flags + kCounter, 1u);
        if (prev == a.epoch * gridDim.x - 1u) {
            __threadfence_system();
            for (int q = 0; q < W; ++q) st_release_sys(a.flags[q] + kDone + a.rank, a.epoch);
        }
        if (blockIdx.x == 0) {
            for (int q = 0; q < W; ++q)
                if (!wait_flag(my_flags + kDone + q, a.epoch, a.budget_ns, 0x0702)) break;
        }
    }
}

}  // namespace fabric
}  // namespace gplk

struct gplk_fabric {
    int rank = 0, world = 0, device = 0, blocks = 0;
    size_t bytes = 0;
    unsigned char* base = nullptr;  // this rank's region: flags, then data
    unsigned char* peer[gplk::fabric::kMaxRanks] = {};
    bool connected = false;
    bool local = false;  // peers are this process's own allocations (no IPC mappings to close)
    unsigned epoch = 0;
};

extern "C" size_t gplk_fabric_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int gplk_fabric_create(int rank, int world, size_t bytes, gplk_fabric** out, void* handle) {
    using namespace gplk;
    if (!out || !handle || world < 1 || world > fabric::kMaxRanks || rank < 0 || rank >= world || bytes == 0 ||
        bytes % 16 != 0)
        return GPLK_STATUS_BAD_ARG;
    *out = nullptr;
    DeviceInfo d;
    int st = require_sm100(&d);
    if (st != GPLK_STATUS_OK) return st;
    gplk_fabric* f = new gplk_fabric();
    f->rank = rank;
    f->world = world;
    f->bytes = bytes;
    cudaGetDevice(&f->device);
    void* p = nullptr;
    if (cudaMalloc(&p, fabric::kFlagBytes + bytes) != cudaSuccess) {
        cudaGetLastError();
        delete f;
        return GPLK_STATUS_CUDA_ERROR;
    }
    f->base = static_cast<unsigned char*>(p);
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, fabric::kFlagBytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        delete f;
        return GPLK_STATUS_CUDA_ERROR;
    }
    memcpy(handle, &h, sizeof(h));
    f->blocks = 2 * d.sm_count;  // two blocks per SM; co-residency is checked by the cooperative launch
    *out = f;
    return GPLK_STATUS_OK;
}

extern "C" int gplk_fabric_connect(gplk_fabric* f, const void* handles) {
    using namespace gplk;
    if (!f || !handles || f->connected) return GPLK_STATUS_BAD_ARG;
    const unsigned char* hs = static_cast<const unsigned char*>(handles);
    for (int q = 0; q < f->world; ++q) {
        if (q == f->rank) {
            f->peer[q] = f->base;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hs + (size_t)q * sizeof(h), sizeof(h));
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            for (int j = 0; j < q; ++j)
                if (j != f->rank && f->peer[j]) cudaIpcCloseMemHandle(f->peer[j]);
            return GPLK_STATUS_CUDA_ERROR;
        }
        f->peer[q] = static_cast<unsigned char*>(p);
    }
    f->connected = true;
    return GPLK_STATUS_OK;
}

extern "C" int gplk_fabric_create_local(int ndev, const int* devices, size_t bytes, gplk_fabric** out) {
    using namespace gplk;
    if (!out || !devices || ndev < 1 || ndev > fabric::kMaxRanks || bytes == 0 || bytes % 16 != 0)
        return GPLK_STATUS_BAD_ARG;
    int cur = 0;
    cudaGetDevice(&cur);
    for (int i = 0; i < ndev; ++i) out[i] = nullptr;
    int st = GPLK_STATUS_OK;
    for (int i = 0; i < ndev && st == GPLK_STATUS_OK; ++i) {
        if (cudaSetDevice(devices[i]) != cudaSuccess) {
            st = GPLK_STATUS_BAD_ARG;
            break;
        }
        DeviceInfo d;
        st = require_sm100(&d);
        if (st != GPLK_STATUS_OK) break;
        gplk_fabric* f = new gplk_fabric();
        f->rank = i;
        f->world = ndev;
        f->bytes = bytes;
        f->device = devices[i];
        f->blocks = 2 * d.sm_count;
        f->local = true;
        void* p = nullptr;
        if (cudaMalloc(&p, fabric::kFlagBytes + bytes) != cudaSuccess ||
            cudaMemset(p, 0, fabric::kFlagBytes) != cudaSuccess) {
            cudaGetLastError();
            if (p) cudaFree(p);
            delete f;
            st = GPLK_STATUS_CUDA_ERROR;
            break;
        }
        f->base = static_cast<unsigned char*>(p);
        out[i] = f;
        for (int j = 0; j < ndev; ++j) {  // peer access to every other device
            if (j == i) continue;
            const cudaError_t e = cudaDeviceEnablePeerAccess(devices[j], 0);
            if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) {
                cudaGetLastError();
                st = GPLK_STATUS_CUDA_ERROR;
                break;
            }
            cudaGetLastError();
        }
    }
    if (st == GPLK_STATUS_OK) {
        for (int i = 0; i < ndev; ++i) {
            for (int q = 0; q < ndev; ++q) out[i]->peer[q] = out[q]->base;
            out[i]->connected = true;
        }
    } else {
        for (int i = 0; i < ndev; ++i) {
            if (!out[i]) continue;
            cudaSetDevice(out[i]->device);
            cudaFree(out[i]->base);
            delete out[i];
            out[i] = nullptr;
        }
    }
    cudaSetDevice(cur);
    return st;
}

extern "C" void* gplk_fabric_data(gplk_fabric* f) { return f ? f->base + gplk::fabric::kFlagBytes : nullptr; }

namespace gplk {
namespace fabric {

template <bool F32>
static const void* kernel_for(int world) {
    switch (world) {
        case 1: return (const void*)allreduce_kernel<1, F32>;
        case 2: return (const void*)allreduce_kernel<2, F32>;
        case 3: return (const void*)allreduce_kernel<3, F32>;
        case 4: return (const void*)allreduce_kernel<4, F32>;
        case 5: return (const void*)allreduce_kernel<5, F32>;
        case 6: return (const void*)allreduce_kernel<6, F32>;
        case 7: return (const void*)allreduce_kernel<7, F32>;
        default: return (const void*)allreduce_kernel<8, F32>;
    }
}

// One in-place allreduce of `n16` 16-byte vectors on this rank's device.
template <bool F32>
static int launch_allreduce(gplk_fabric* f, size_t n16, cudaStream_t stream) {
    Args a;
    memset(&a, 0, sizeof(a));
    for (int q = 0; q < f->world; ++q) {
        a.src[q] = reinterpret_cast<const uint4*>(f->peer[q] + kFlagBytes);
        a.dst[q] = reinterpret_cast<uint4*>(f->peer[q] + kFlagBytes);
        a.flags[q] = reinterpret_cast<unsigned*>(f->peer[q]);
    }
    a.rank = f->rank;
    a.world = f->world;
    a.n16 = n16;
    a.chunk16 = (n16 + (size_t)f->world - 1) / (size_t)f->world;
    a.epoch = ++f->epoch;
    a.budget_ns = 2000000000ull;
    void* args[] = {&a};
    // The launch goes to the fabric's device (a single process may drive several).
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != f->device) cudaSetDevice(f->device);
    const cudaError_t e = cudaLaunchCooperativeKernel(kernel_for<F32>(f->world), dim3((unsigned)f->blocks),
                                                      dim3(kThreads), args, 0, stream);
    if (cur != f->device) cudaSetDevice(cur);
    return launch_status(e);
}

}  // namespace fabric
}  // namespace gplk

extern "C" int gplk_fabric_allreduce_f32(gplk_fabric* f, size_t count, cudaStream_t stream) {
    using namespace gplk;
    if (!f || !f->connected || count % 4 != 0 || count * 4 > f->bytes) return GPLK_STATUS_BAD_ARG;
    if (count == 0) return GPLK_STATUS_OK;
    return fabric::launch_allreduce<true>(f, count / 4, stream);
}

extern "C" int gplk_fabric_allreduce_bf16(gplk_fabric* f, size_t count, cudaStream_t stream) {
    using namespace gplk;
    if (!f || !f->connected || count % 8 != 0 || count * 2 > f->bytes) return GPLK_STATUS_BAD_ARG;
    if (count == 0) return GPLK_STATUS_OK;
    return fabric::launch_allreduce<false>(f, count / 8, stream);
}

extern "C" int gplk_fabric_destroy(gplk_fabric* f) {
    if (!f) return GPLK_STATUS_OK;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaSetDevice(f->device);
    if (!f->local)
        for (int q = 0; q < f->world; ++q)
            if (q != f->rank && f->peer[q]) cudaIpcCloseMemHandle(f->peer[q]);
    if (f->base) cudaFree(f->base);
    cudaSetDevice(dev);
    delete f;
    return GPLK_STATUS_OK;
}
