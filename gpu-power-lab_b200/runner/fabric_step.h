/*
 * fabric_step.h - the per-cycle fabric step of the multi-GPU powervirus rung:
 * a BF16 sum allreduce across the runner processes of one node (one process
 * per GPU, all in phase), issued on the burst's stream right after every
 * duty-cycle burst.
 *
 * The reference's runner has no such step: its powervirus duty loop
 * (runner/src/workload_powervirus.cu:603-647) only bursts and sleeps, and its
 * collectives live in a separate rung (runner/src/workload_nccl.cu:119-291,
 * ncclAllReduce over ncclCommInitAll devices). The CLI parser is kept as it
 * is, so the step is configured by environment variables, read once at
 * set-up:
 *
 *   GPL_FABRIC          "gplk" (gplk_fabric_allreduce_bf16: one kernel over
 *                       NVLink peer memory) or "nccl" (ncclAllReduce, BF16,
 *                       sum); unset or empty: no fabric step
 *   GPL_FABRIC_WORLD    number of runner processes (1..8)
 *   GPL_FABRIC_RANK     this process's rank, 0..world-1
 *   GPL_FABRIC_DIR      rendezvous directory, shared by the processes and
 *                       empty at the start of each job: rank r writes its
 *                       CUDA IPC handle (gplk) or rank 0 the NCCL unique id
 *                       there, and every rank waits for the others' files
 *   GPL_FABRIC_MIB      allreduce size in MiB of BF16 (default 256)
 *   GPL_FABRIC_TIMEOUT_S  bound on the rendezvous wait (default 60)
 *
 * Every cycle refreshes the allreduce buffer from a pristine copy (a device
 * copy, so values stay those of the first cycle, as an out-of-place
 * collective would leave them), then reduces it. The allreduce alone is
 * timed with CUDA events on the stream. A rank that never arrives makes the
 * gplk step return GPLK_STATUS_DEVICE_TIMEOUT (bounded 2 s waits in the
 * kernel); the fabric must then be torn down, not reused.
 */
#ifndef GPL_FABRIC_STEP_H
#define GPL_FABRIC_STEP_H

#include <cuda_runtime_api.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int active;                  /* a fabric step ran this process */
    const char *impl;            /* "gplk" or "nccl" */
    int rank, world;
    size_t bytes;                /* allreduce size per rank */
    unsigned long long cycles;   /* allreduces timed */
    double median_ms, max_ms;    /* allreduce time per cycle (CUDA events) */
    double busbw_gbs;            /* 2 (N-1)/N x bytes / median time */
} gpl_fabric_stats_t;

/* Reads the environment and sets the step up on the current device (the
 * rendezvous may wait for the other ranks), then runs one untimed step on
 * every rank. Returns 0 with no fabric requested or when set up; -1 with
 * *err set (static string) otherwise. */
int gpl_fabric_step_init(const char **err);

/* True once gpl_fabric_step_init has set a step up. */
int gpl_fabric_step_enabled(void);

/* Enqueues one cycle's step on `stream` (refresh, then the allreduce between
 * two events). Asynchronous; 0 or -1. */
int gpl_fabric_step_enqueue(cudaStream_t stream);

/* After the stream has synchronised: records the last step's time. */
void gpl_fabric_step_record(void);

/* Frees the step's buffers and communicator. Stats stay readable. */
void gpl_fabric_step_free(void);

/* The stats of this process's fabric steps (active == 0 when none ran). */
const gpl_fabric_stats_t *gpl_fabric_stats(void);

/* Pure host helpers, exported for the host tests. */
double gpl_fabric_busbw_gbs(size_t bytes, double seconds, int world);
double gpl_fabric_median(double *v, size_t n); /* sorts v in place */
/* Exchanges `len` bytes per rank through files dir/<tag>.<rank>; `all`
 * receives world x len bytes in rank order. 0, or -1 after timeout_s. */
int gpl_fabric_rendezvous(const char *dir, const char *tag, int rank, int world, const void *mine, size_t len,
                          void *all, double timeout_s);
/* Whole duty cycles that fit the steady window (at least one), the same on
 * every rank, so every rank takes the same number of fabric steps. */
unsigned long long gpl_fabric_cycles(double steady_s, double on_ms, double off_ms);

#ifdef __cplusplus
}
#endif

#endif /* GPL_FABRIC_STEP_H */
