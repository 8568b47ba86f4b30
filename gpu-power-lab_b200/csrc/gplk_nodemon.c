/* gplk_nodemon.c - node-level power telemetry (include/gplk_nodemon.h).
 *
 * One pthread per device. Each thread polls, at the requested rate on an
 * absolute-deadline schedule (clock_nanosleep, so wake-up jitter does not
 * accumulate), the driver-averaged power and the instantaneous power field,
 * and every drain period pulls the driver's buffered power samples newer than
 * the last one it has seen. Samples go into a per-device growable array under
 * a mutex. All timestamps are on the host's CLOCK_REALTIME microsecond base,
 * which is also the base of the driver's sample timestamps, so polled and
 * buffered samples of every device share one timebase.
 */
#define _GNU_SOURCE
#include "../../include/gplk_nodemon.h"

#include <dlfcn.h>
#include <nvml.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#define GPLK_NODEMON_MAX_DEV 64

/* The NVML entry points used, resolved by name from the loaded library. */
typedef struct {
    void *lib;
    nvmlReturn_t (*init)(void);
    nvmlReturn_t (*shutdown)(void);
    nvmlReturn_t (*handle_by_index)(unsigned int, nvmlDevice_t *);
    nvmlReturn_t (*power_usage)(nvmlDevice_t, unsigned int *);
    nvmlReturn_t (*field_values)(nvmlDevice_t, int, nvmlFieldValue_t *);
    nvmlReturn_t (*samples)(nvmlDevice_t, nvmlSamplingType_t, unsigned long long, nvmlValueType_t *,
                            unsigned int *, nvmlSample_t *);
} nvml_api;

typedef struct {
    gplk_power_sample *v;
    size_t n, cap;
} sample_vec;

typedef struct {
    struct gplk_nodemon *m;
    int index;           /* NVML device index */
    nvmlDevice_t dev;
    pthread_t thread;
    int started;
    sample_vec s;
    unsigned long long last_ts; /* newest buffered-sample timestamp seen */
    nvmlSample_t *buf;          /* drain scratch */
    unsigned int buf_cap;
} dev_state;

struct gplk_nodemon {
    nvml_api api;
    int ndev;
    int sample_hz, drain_ms;
    int64_t t0_us; /* CLOCK_REALTIME at open */
    volatile int stop;
    pthread_mutex_t mu;
    dev_state d[GPLK_NODEMON_MAX_DEV];
};

static int64_t realtime_us(void) {
    struct timespec ts;
    clock_gettime(CLOCK_REALTIME, &ts);
    return (int64_t)ts.tv_sec * 1000000 + ts.tv_nsec / 1000;
}

static void push(gplk_nodemon *m, dev_state *d, const gplk_power_sample *x) {
    pthread_mutex_lock(&m->mu);
    if (d->s.n == d->s.cap) {
        size_t cap = d->s.cap ? d->s.cap * 2 : 4096;
        gplk_power_sample *nv = (gplk_power_sample *)realloc(d->s.v, cap * sizeof(*nv));
        if (!nv) {
            pthread_mutex_unlock(&m->mu);
            return; /* out of host memory: drop the sample */
        }
        d->s.v = nv;
        d->s.cap = cap;
    }
    d->s.v[d->s.n++] = *x;
    pthread_mutex_unlock(&m->mu);
}

static double value_watts(nvmlValueType_t t, nvmlValue_t v) {
    switch (t) {
        case NVML_VALUE_TYPE_DOUBLE: return v.dVal / 1000.0;
        case NVML_VALUE_TYPE_UNSIGNED_LONG: return (double)v.ulVal / 1000.0;
        case NVML_VALUE_TYPE_UNSIGNED_LONG_LONG: return (double)v.ullVal / 1000.0;
        case NVML_VALUE_TYPE_SIGNED_LONG_LONG: return (double)v.sllVal / 1000.0;
        case NVML_VALUE_TYPE_SIGNED_INT: return (double)v.siVal / 1000.0;
        default: return (double)v.uiVal / 1000.0; /* milliwatts as unsigned int */
    }
}

static void drain(gplk_nodemon *m, dev_state *d) {
    nvmlValueType_t vt;
    unsigned int count = 0;
    nvmlReturn_t r = m->api.samples(d->dev, NVML_TOTAL_POWER_SAMPLES, d->last_ts, &vt, &count, NULL);
    if ((r != NVML_SUCCESS && r != NVML_ERROR_INSUFFICIENT_SIZE) || count == 0) return;
    if (count > d->buf_cap) {
        nvmlSample_t *nb = (nvmlSample_t *)realloc(d->buf, (size_t)count * sizeof(*nb));
        if (!nb) return;
        d->buf = nb;
        d->buf_cap = count;
    }
    if (m->api.samples(d->dev, NVML_TOTAL_POWER_SAMPLES, d->last_ts, &vt, &count, d->buf) != NVML_SUCCESS) return;
    for (unsigned int i = 0; i < count; ++i) {
        const unsigned long long ts = d->buf[i].timeStamp;
        if (ts <= d->last_ts) continue;
        gplk_power_sample x;
        x.t_s = (double)((int64_t)ts - m->t0_us) / 1e6;
        x.power_w = (float)value_watts(vt, d->buf[i].sampleValue);
        x.instant_w = -1.0f;
        x.device = d->index;
        x.source = GPLK_NODEMON_BUFFERED;
        push(m, d, &x);
    }
    for (unsigned int i = 0; i < count; ++i)
        if (d->buf[i].timeStamp > d->last_ts) d->last_ts = d->buf[i].timeStamp;
}

static void *sampler(void *arg) {
    dev_state *d = (dev_state *)arg;
    gplk_nodemon *m = d->m;
    const long period_ns = 1000000000L / m->sample_hz;
    struct timespec next;
    clock_gettime(CLOCK_MONOTONIC, &next);
    int64_t last_drain = realtime_us();
    while (!m->stop) {
        gplk_power_sample x;
        unsigned int mw = 0;
        const int64_t now = realtime_us();
        x.power_w = m->api.power_usage(d->dev, &mw) == NVML_SUCCESS ? (float)mw / 1000.0f : -1.0f;
        x.instant_w = -1.0f;
        if (m->api.field_values) {
            nvmlFieldValue_t fv;
            memset(&fv, 0, sizeof(fv));
            fv.fieldId = NVML_FI_DEV_POWER_INSTANT;
            if (m->api.field_values(d->dev, 1, &fv) == NVML_SUCCESS && fv.nvmlReturn == NVML_SUCCESS)
                x.instant_w = (float)value_watts(fv.valueType, fv.value);
        }
        x.t_s = (double)(now - m->t0_us) / 1e6;
        x.device = d->index;
        x.source = GPLK_NODEMON_POLLED;
        if (x.power_w >= 0.0f) push(m, d, &x);
        if (m->drain_ms > 0 && m->api.samples && now - last_drain >= (int64_t)m->drain_ms * 1000) {
            drain(m, d);
            last_drain = now;
        }
        next.tv_nsec += period_ns;
        while (next.tv_nsec >= 1000000000L) {
            next.tv_nsec -= 1000000000L;
            next.tv_sec += 1;
        }
        clock_nanosleep(CLOCK_MONOTONIC, TIMER_ABSTIME, &next, NULL);
    }
    if (m->drain_ms > 0 && m->api.samples) drain(m, d); /* the tail of the buffer */
    return NULL;
}

static void *sym(void *lib, const char *name) { return dlsym(lib, name); }

int gplk_nodemon_open(const char *nvml_path, int ndev, const int *devices, int sample_hz, int drain_ms,
                      gplk_nodemon **out) {
    if (!out || ndev < 1 || ndev > GPLK_NODEMON_MAX_DEV || !devices || sample_hz < 1 || sample_hz > 1000 ||
        drain_ms < 0)
        return -1;
    *out = NULL;
    gplk_nodemon *m = (gplk_nodemon *)calloc(1, sizeof(*m));
    if (!m) return -1;
    m->api.lib = dlopen(nvml_path ? nvml_path : "libnvidia-ml.so.1", RTLD_NOW | RTLD_LOCAL);
    if (!m->api.lib) {
        free(m);
        return -2;
    }
    m->api.init = (nvmlReturn_t(*)(void))sym(m->api.lib, "nvmlInit_v2");
    m->api.shutdown = (nvmlReturn_t(*)(void))sym(m->api.lib, "nvmlShutdown");
    m->api.handle_by_index = (nvmlReturn_t(*)(unsigned int, nvmlDevice_t *))sym(m->api.lib,
                                                                               "nvmlDeviceGetHandleByIndex_v2");
    m->api.power_usage = (nvmlReturn_t(*)(nvmlDevice_t, unsigned int *))sym(m->api.lib, "nvmlDeviceGetPowerUsage");
    m->api.field_values =
        (nvmlReturn_t(*)(nvmlDevice_t, int, nvmlFieldValue_t *))sym(m->api.lib, "nvmlDeviceGetFieldValues");
    m->api.samples = (nvmlReturn_t(*)(nvmlDevice_t, nvmlSamplingType_t, unsigned long long, nvmlValueType_t *,
                                      unsigned int *, nvmlSample_t *))sym(m->api.lib, "nvmlDeviceGetSamples");
    if (!m->api.init || !m->api.shutdown || !m->api.handle_by_index || !m->api.power_usage ||
        m->api.init() != NVML_SUCCESS) {
        dlclose(m->api.lib);
        free(m);
        return -2;
    }
    pthread_mutex_init(&m->mu, NULL);
    m->ndev = ndev;
    m->sample_hz = sample_hz;
    m->drain_ms = drain_ms;
    m->t0_us = realtime_us();
    for (int i = 0; i < ndev; ++i) {
        dev_state *d = &m->d[i];
        d->m = m;
        d->index = devices[i];
        if (devices[i] < 0 || m->api.handle_by_index((unsigned int)devices[i], &d->dev) != NVML_SUCCESS) {
            gplk_nodemon_close(m);
            return -3;
        }
        /* Start the buffered path at "now": older driver samples predate the monitor. */
        d->last_ts = (unsigned long long)m->t0_us;
    }
    for (int i = 0; i < ndev; ++i) {
        if (pthread_create(&m->d[i].thread, NULL, sampler, &m->d[i]) != 0) {
            gplk_nodemon_close(m);
            return -1;
        }
        m->d[i].started = 1;
    }
    *out = m;
    return 0;
}

int gplk_nodemon_stop(gplk_nodemon *m) {
    if (!m) return -1;
    m->stop = 1;
    for (int i = 0; i < m->ndev; ++i) {
        if (m->d[i].started) {
            pthread_join(m->d[i].thread, NULL);
            m->d[i].started = 0;
        }
    }
    return 0;
}

size_t gplk_nodemon_count(gplk_nodemon *m) {
    if (!m) return 0;
    size_t n = 0;
    pthread_mutex_lock(&m->mu);
    for (int i = 0; i < m->ndev; ++i) n += m->d[i].s.n;
    pthread_mutex_unlock(&m->mu);
    return n;
}

static int by_time(const void *a, const void *b) {
    const double x = ((const gplk_power_sample *)a)->t_s, y = ((const gplk_power_sample *)b)->t_s;
    return x < y ? -1 : x > y ? 1 : 0;
}

size_t gplk_nodemon_read(gplk_nodemon *m, gplk_power_sample *out, size_t max) {
    if (!m || !out) return 0;
    size_t k = 0;
    pthread_mutex_lock(&m->mu);
    for (int i = 0; i < m->ndev && k < max; ++i) {
        const size_t n = m->d[i].s.n < max - k ? m->d[i].s.n : max - k;
        memcpy(out + k, m->d[i].s.v, n * sizeof(*out));
        /* buffered samples arrive in batches after the polled ones: order by time */
        qsort(out + k, n, sizeof(*out), by_time);
        k += n;
    }
    pthread_mutex_unlock(&m->mu);
    return k;
}

size_t gplk_nodemon_node_series(gplk_nodemon *m, int source, double t0_s, double bin_s, double *w_out, size_t max) {
    if (!m || !w_out || max == 0 || !(bin_s > 0.0)) return 0;
    double *sum = (double *)calloc(max, sizeof(double));
    double *dev_sum = (double *)calloc(max, sizeof(double));
    int *dev_cnt = (int *)calloc(max, sizeof(int));
    if (!sum || !dev_sum || !dev_cnt) {
        free(sum);
        free(dev_sum);
        free(dev_cnt);
        return 0;
    }
    size_t nbins = 0;
    pthread_mutex_lock(&m->mu);
    for (int i = 0; i < m->ndev; ++i) {
        memset(dev_sum, 0, max * sizeof(double));
        memset(dev_cnt, 0, max * sizeof(int));
        const sample_vec *s = &m->d[i].s;
        for (size_t j = 0; j < s->n; ++j) {
            const gplk_power_sample *x = &s->v[j];
            if (x->source != source || x->t_s < t0_s) continue;
            const size_t b = (size_t)((x->t_s - t0_s) / bin_s);
            if (b >= max) continue;
            dev_sum[b] += x->power_w;
            dev_cnt[b] += 1;
            if (b + 1 > nbins) nbins = b + 1;
        }
        double carry = 0.0;
        for (size_t b = 0; b < max; ++b) {
            if (dev_cnt[b]) carry = dev_sum[b] / dev_cnt[b];
            sum[b] += carry;
        }
    }
    pthread_mutex_unlock(&m->mu);
    memcpy(w_out, sum, nbins * sizeof(double));
    free(sum);
    free(dev_sum);
    free(dev_cnt);
    return nbins;
}

int gplk_nodemon_close(gplk_nodemon *m) {
    if (!m) return 0;
    gplk_nodemon_stop(m);
    for (int i = 0; i < m->ndev; ++i) {
        free(m->d[i].s.v);
        free(m->d[i].buf);
    }
    if (m->api.shutdown) m->api.shutdown();
    if (m->api.lib) dlclose(m->api.lib);
    pthread_mutex_destroy(&m->mu);
    free(m);
    return 0;
}
