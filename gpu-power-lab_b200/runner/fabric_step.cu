/*
 * fabric_step.cu - the per-cycle fabric step of the multi-GPU powervirus
 * rung (see fabric_step.h): set-up through a file rendezvous between the
 * runner processes of one node, one BF16 sum allreduce per duty cycle
 * (libgplk's NVLink peer-memory kernel, or NCCL), per-cycle timing.
 *
 * Host code only; the allreduce kernel is gplk_fabric_allreduce_bf16 in
 * libgplk. No multicast of any kind.
 */
#include "fabric_step.h"

#include <cuda_runtime.h>
#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <vector>

#include "gplk.h"

#ifdef GPL_HAVE_NCCL
#include <nccl.h>
#endif

namespace {

struct Step {
    bool enabled = false;
    bool use_nccl = false;
    gplk_fabric *fab = nullptr;
    void *pristine = nullptr;  // the cycle's input, copied into the buffer each cycle
    void *recv = nullptr;      // NCCL output buffer
    size_t bytes = 0;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    bool pending = false;
    std::vector<double> ms;
#ifdef GPL_HAVE_NCCL
    ncclComm_t comm = nullptr;
#endif
};

Step g_step;
gpl_fabric_stats_t g_stats;

double now_s() {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

int env_int(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

}  // namespace

extern "C" {

double gpl_fabric_busbw_gbs(size_t bytes, double seconds, int world) {
    if (seconds <= 0.0 || world < 1) return 0.0;
    return 2.0 * (double)(world - 1) / (double)world * (double)bytes / seconds / 1e9;
}

double gpl_fabric_median(double *v, size_t n) {
    if (n == 0) return 0.0;
    std::sort(v, v + n);
    return (n % 2) ? v[n / 2] : 0.5 * (v[n / 2 - 1] + v[n / 2]);
}

/* Exchange `len` bytes between `world` processes through files in `dir`:
 * writes this rank's bytes to dir/<tag>.<rank> (through a temporary file and
 * a rename, so a reader never sees a partial file), then waits until every
 * rank's file holds `len` bytes and reads them, in rank order, into `all`
 * (world x len bytes). Returns 0, or -1 after timeout_s or on an I/O error. */
int gpl_fabric_rendezvous(const char *dir, const char *tag, int rank, int world, const void *mine, size_t len,
                          void *all, double timeout_s) {
    if (!dir || !tag || rank < 0 || rank >= world || (len && (!mine || !all))) return -1;
    char path[4096], tmp[4096];
    snprintf(path, sizeof path, "%s/%s.%d", dir, tag, rank);
    snprintf(tmp, sizeof tmp, "%s/.%s.%d.tmp", dir, tag, rank);
    FILE *f = fopen(tmp, "wb");
    if (!f) return -1;
    const bool wrote = len == 0 || fwrite(mine, 1, len, f) == len;
    if (fclose(f) != 0 || !wrote || rename(tmp, path) != 0) return -1;
    const double t0 = now_s();
    for (int q = 0; q < world; ++q) {
        snprintf(path, sizeof path, "%s/%s.%d", dir, tag, q);
        while (true) {
            struct stat sb;
            if (stat(path, &sb) == 0 && (size_t)sb.st_size == len) break;
            if (now_s() - t0 > timeout_s) return -1;
            usleep(2000);
        }
        if (len) {
            FILE *r = fopen(path, "rb");
            if (!r) return -1;
            const size_t got = fread((char *)all + (size_t)q * len, 1, len, r);
            fclose(r);
            if (got != len) return -1;
        }
    }
    return 0;
}

/* Whole duty cycles (burst + fabric step + idle) that fit in the steady
 * window, at least one: every rank computes the same count, so all of them
 * take the same number of fabric steps. */
unsigned long long gpl_fabric_cycles(double steady_s, double on_ms, double off_ms) {
    const double period_s = (on_ms + off_ms) / 1e3;
    if (period_s <= 0.0) return 1;
    const double c = steady_s / period_s;
    return c < 1.0 ? 1ull : (unsigned long long)(c + 1e-9);
}

int gpl_fabric_step_init(const char **err) {
    static const char *e_cfg = "fabric step: GPL_FABRIC_WORLD / GPL_FABRIC_RANK / GPL_FABRIC_DIR missing or invalid";
    static const char *e_impl = "fabric step: GPL_FABRIC must be gplk or nccl";
    static const char *e_alloc = "fabric step: out of memory";
    static const char *e_rdv = "fabric step: rendezvous with the other ranks timed out";
    static const char *e_conn = "fabric step: connecting to the peers' buffers failed";
    static const char *e_comm = "fabric step: NCCL communicator set-up failed";
    memset(&g_stats, 0, sizeof g_stats);
    const char *impl = getenv("GPL_FABRIC");
    if (!impl || !*impl) return 0;
    const bool nccl = !strcmp(impl, "nccl");
    if (!nccl && strcmp(impl, "gplk")) {
        *err = e_impl;
        return -1;
    }
    const int world = env_int("GPL_FABRIC_WORLD", 0), rank = env_int("GPL_FABRIC_RANK", -1);
    const char *dir = getenv("GPL_FABRIC_DIR");
    const double timeout_s = (double)env_int("GPL_FABRIC_TIMEOUT_S", 60);
    const int mib = env_int("GPL_FABRIC_MIB", 256);
    if (world < 1 || world > 8 || rank < 0 || rank >= world || !dir || !*dir || mib <= 0) {
        *err = e_cfg;
        return -1;
    }
    Step &s = g_step;
    s.bytes = (size_t)mib << 20;
    s.use_nccl = nccl;
    if (cudaMalloc(&s.pristine, s.bytes) != cudaSuccess || cudaMemset(s.pristine, 0x3c, s.bytes) != cudaSuccess ||
        cudaEventCreate(&s.ev0) != cudaSuccess || cudaEventCreate(&s.ev1) != cudaSuccess) {
        cudaGetLastError();
        *err = e_alloc;
        gpl_fabric_step_free();
        return -1;
    }
    if (nccl) {
#ifdef GPL_HAVE_NCCL
        ncclUniqueId id;
        memset(&id, 0, sizeof id);  // ranks other than 0 publish zeros; rank 0's id is the one used
        if (rank == 0 && ncclGetUniqueId(&id) != ncclSuccess) {
            *err = e_comm;
            gpl_fabric_step_free();
            return -1;
        }
        std::vector<unsigned char> ids((size_t)world * sizeof id);
        if (gpl_fabric_rendezvous(dir, "nccl", rank, world, &id, sizeof id, ids.data(), timeout_s) != 0) {
            *err = e_rdv;
            gpl_fabric_step_free();
            return -1;
        }
        memcpy(&id, ids.data(), sizeof id);  // rank 0's id
        if (cudaMalloc(&s.recv, s.bytes) != cudaSuccess) {
            cudaGetLastError();
            *err = e_alloc;
            gpl_fabric_step_free();
            return -1;
        }
        if (ncclCommInitRank(&s.comm, world, id, rank) != ncclSuccess) {
            s.comm = nullptr;
            *err = e_comm;
            gpl_fabric_step_free();
            return -1;
        }
#else
        *err = "fabric step: this runner was built without NCCL";
        gpl_fabric_step_free();
        return -1;
#endif
    } else {
        const size_t hb = gplk_fabric_handle_bytes();
        std::vector<unsigned char> mine(hb), all((size_t)world * hb);
        if (gplk_fabric_create(rank, world, s.bytes, &s.fab, mine.data()) != GPLK_STATUS_OK) {
            s.fab = nullptr;
            *err = e_alloc;
            gpl_fabric_step_free();
            return -1;
        }
        if (gpl_fabric_rendezvous(dir, "gplk", rank, world, mine.data(), hb, all.data(), timeout_s) != 0) {
            *err = e_rdv;
            gpl_fabric_step_free();
            return -1;
        }
        if (gplk_fabric_connect(s.fab, all.data()) != GPLK_STATUS_OK) {
            *err = e_conn;
            gpl_fabric_step_free();
            return -1;
        }
        // Every rank mapped every peer before anyone's first allreduce.
        if (gpl_fabric_rendezvous(dir, "gplk-ready", rank, world, nullptr, 0, nullptr, timeout_s) != 0) {
            *err = e_rdv;
            gpl_fabric_step_free();
            return -1;
        }
    }
    s.enabled = true;
    g_stats.impl = nccl ? "nccl" : "gplk";
    g_stats.rank = rank;
    g_stats.world = world;
    g_stats.bytes = s.bytes;
    // One untimed step, on every rank at the same point: the first launch of
    // the allreduce (module load, NCCL's first collective) happens here, not
    // inside the first cycle's timing.
    {
        cudaStream_t ws = nullptr;
        const bool ok = cudaStreamCreateWithFlags(&ws, cudaStreamNonBlocking) == cudaSuccess &&
                        gpl_fabric_step_enqueue(ws) == 0 && cudaStreamSynchronize(ws) == cudaSuccess;
        if (ws) cudaStreamDestroy(ws);
        s.pending = false;
        int code = 0, site = 0;
        if (!ok || gplk_status_read(&code, &site, 1) != GPLK_STATUS_OK || code != GPLK_STATUS_OK) {
            cudaGetLastError();
            *err = "fabric step: the warm-up allreduce failed";
            gpl_fabric_step_free();
            return -1;
        }
    }
    return 0;
}

int gpl_fabric_step_enabled(void) { return g_step.enabled ? 1 : 0; }

int gpl_fabric_step_enqueue(cudaStream_t stream) {
    Step &s = g_step;
    if (!s.enabled) return 0;
    const size_t count = s.bytes / 2;  // BF16 elements
    if (s.use_nccl) {
#ifdef GPL_HAVE_NCCL
        if (cudaEventRecord(s.ev0, stream) != cudaSuccess) return -1;
        if (ncclAllReduce(s.pristine, s.recv, count, ncclBfloat16, ncclSum, s.comm, stream) != ncclSuccess)
            return -1;
#else
        return -1;
#endif
    } else {
        void *buf = gplk_fabric_data(s.fab);
        if (cudaMemcpyAsync(buf, s.pristine, s.bytes, cudaMemcpyDeviceToDevice, stream) != cudaSuccess) return -1;
        if (cudaEventRecord(s.ev0, stream) != cudaSuccess) return -1;
        if (gplk_fabric_allreduce_bf16(s.fab, count, stream) != GPLK_STATUS_OK) return -1;
    }
    if (cudaEventRecord(s.ev1, stream) != cudaSuccess) return -1;
    s.pending = true;
    return 0;
}

void gpl_fabric_step_record(void) {
    Step &s = g_step;
    if (!s.pending) return;
    s.pending = false;
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, s.ev0, s.ev1) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    s.ms.push_back((double)ms);
    std::vector<double> v(s.ms);
    g_stats.active = 1;
    g_stats.cycles = (unsigned long long)v.size();
    g_stats.max_ms = *std::max_element(v.begin(), v.end());
    g_stats.median_ms = gpl_fabric_median(v.data(), v.size());
    g_stats.busbw_gbs = gpl_fabric_busbw_gbs(s.bytes, g_stats.median_ms / 1e3, g_stats.world);
}

void gpl_fabric_step_free(void) {
    Step &s = g_step;
#ifdef GPL_HAVE_NCCL
    if (s.comm) ncclCommDestroy(s.comm);
    s.comm = nullptr;
#endif
    if (s.fab) gplk_fabric_destroy(s.fab);
    if (s.pristine) cudaFree(s.pristine);
    if (s.recv) cudaFree(s.recv);
    if (s.ev0) cudaEventDestroy(s.ev0);
    if (s.ev1) cudaEventDestroy(s.ev1);
    s.fab = nullptr;
    s.pristine = s.recv = nullptr;
    s.ev0 = s.ev1 = nullptr;
    s.enabled = false;
    s.pending = false;
}

const gpl_fabric_stats_t *gpl_fabric_stats(void) { return &g_stats; }

}  // extern "C"
