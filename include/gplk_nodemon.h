/* gplk_nodemon.h - node-level power telemetry: one sampler thread per GPU of
 * the node, in one process, on a shared host timebase.
 *
 * The reference's runner samples one device per process (its NVML sampler
 * thread, runner/src/telemetry.c:83-258) by polling nvmlDeviceGetPowerUsage
 * and the NVML_FI_DEV_POWER_INSTANT field; its design notes name two further
 * paths it did not build (sections "Instrumenting transients" and
 * "Multi-GPU and multi-node phase alignment"): draining the
 * driver's buffered power samples with
 * nvmlDeviceGetSamples(NVML_TOTAL_POWER_SAMPLES), which carry their own
 * timestamps, and the node-level sum of all GPUs swinging in phase versus
 * deliberately staggered. This library does both. It only reads NVML: it
 * changes no limit, clock or mode.
 *
 * NVML is loaded with dlopen (default "libnvidia-ml.so.1"), so a caller or a
 * test can point it at another implementation of the same functions. No
 * counterpart in the reference's C API; include/gplk.h is independent of it.
 */
#ifndef GPLK_NODEMON_H
#define GPLK_NODEMON_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    GPLK_NODEMON_POLLED = 0,  /* nvmlDeviceGetPowerUsage (driver-averaged) + POWER_INSTANT, host timestamp */
    GPLK_NODEMON_BUFFERED = 1 /* nvmlDeviceGetSamples(NVML_TOTAL_POWER_SAMPLES), driver timestamp */
};

typedef struct {
    double t_s;        /* seconds since the monitor started, host CLOCK_REALTIME base */
    float power_w;     /* polled: driver-averaged power; buffered: the buffered sample */
    float instant_w;   /* polled: NVML_FI_DEV_POWER_INSTANT, or -1 when unsupported; buffered: -1 */
    int device;        /* NVML device index */
    int source;        /* GPLK_NODEMON_POLLED or GPLK_NODEMON_BUFFERED */
} gplk_power_sample;

typedef struct gplk_nodemon gplk_nodemon;

/* Start one sampler thread per listed NVML device index, polling at
 * sample_hz (1..1000) and draining the driver's sample buffer every
 * `drain_ms` (0 disables the buffered path). nvml_path NULL loads
 * "libnvidia-ml.so.1". Returns 0 on success, -1 on bad arguments, -2 when
 * NVML cannot be loaded or initialised, -3 when a device cannot be opened. */
int gplk_nodemon_open(const char *nvml_path, int ndev, const int *devices, int sample_hz, int drain_ms,
                      gplk_nodemon **out);

/* Stop the threads (samples stay readable until gplk_nodemon_close). */
int gplk_nodemon_stop(gplk_nodemon *m);

/* Samples taken so far (both sources). */
size_t gplk_nodemon_count(gplk_nodemon *m);

/* Copy up to `max` samples, device by device, each device's in time order.
 * Returns the number copied. Safe while the threads run. */
size_t gplk_nodemon_read(gplk_nodemon *m, gplk_power_sample *out, size_t max);

/* The node-level power series: the samples of `source` binned into windows
 * of bin_s seconds from t0_s; in each bin, each device contributes the mean
 * of its samples in the bin (a device with none carries its previous value
 * forward, 0 before its first sample), and the bin's value is the sum over
 * devices. Writes up to `max` bins to w_out (watts), returns the count. */
size_t gplk_nodemon_node_series(gplk_nodemon *m, int source, double t0_s, double bin_s, double *w_out, size_t max);

/* Stop if needed, release NVML and free everything. */
int gplk_nodemon_close(gplk_nodemon *m);

#ifdef __cplusplus
}
#endif

#endif /* GPLK_NODEMON_H */
