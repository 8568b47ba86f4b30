/*
 * gpl_fault.h - host-side fault injection for the drop-in workloads, so the
 * runner's error path (result "oom" / "cuda_error", exit 5) can be tested
 * without making a GPU fault. Off unless GPL_FAULT is set:
 *   GPL_FAULT=alloc   the workload fails as a device allocation would
 *   GPL_FAULT=launch  the workload fails as a kernel launch would
 */
#ifndef GPL_FAULT_H
#define GPL_FAULT_H

#include <stdlib.h>
#include <string.h>

static inline int gpl_fault_is(const char *what) {
    const char *f = getenv("GPL_FAULT");
    return f != NULL && strcmp(f, what) == 0;
}

#define GPL_FAULT_ALLOC_MSG "out of memory (injected by GPL_FAULT=alloc)"
#define GPL_FAULT_LAUNCH_MSG "kernel launch failed (injected by GPL_FAULT=launch)"

#endif
