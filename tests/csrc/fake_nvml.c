/* fake_nvml.c - a stand-in for the few NVML functions libgplk_nodemon.so
 * loads, for CPU tests. TEST INFRASTRUCTURE, built by tests/test_nodemon.py.
 * Power is a square wave on the host clock: FAKE_NVML_PERIOD_MS (default
 * 200), FAKE_NVML_HIGH_W / FAKE_NVML_LOW_W (default 900 / 300) for the first
 * / second half of each period. With FAKE_NVML_STAGGER=1 device i is shifted
 * by i * period / FAKE_NVML_NDEV (default 2). The instantaneous field reads
 * 50 W above the averaged value. The driver sample buffer holds one sample
 * every 20 ms on the same clock. Devices 0..7 exist. */
#include <nvml.h>
#include <stdint.h>
#include <stdlib.h>
#include <time.h>

static double envd(const char *k, double d) {
    const char *v = getenv(k);
    return v && *v ? atof(v) : d;
}

static int64_t now_us(void) {
    struct timespec ts;
    clock_gettime(CLOCK_REALTIME, &ts);
    return (int64_t)ts.tv_sec * 1000000 + ts.tv_nsec / 1000;
}

static double watts_at(int dev, int64_t t_us) {
    const double period = envd("FAKE_NVML_PERIOD_MS", 200.0) * 1000.0;
    const double shift = envd("FAKE_NVML_STAGGER", 0.0) > 0.5 ? dev * period / envd("FAKE_NVML_NDEV", 2.0) : 0.0;
    double ph = (double)t_us - shift;
    ph = ph - period * (double)(int64_t)(ph / period);
    if (ph < 0) ph += period;
    return ph < period / 2 ? envd("FAKE_NVML_HIGH_W", 900.0) : envd("FAKE_NVML_LOW_W", 300.0);
}

static int dev_of(nvmlDevice_t d) { return (int)((uintptr_t)d) - 1; }

nvmlReturn_t nvmlInit_v2(void) { return NVML_SUCCESS; }
nvmlReturn_t nvmlShutdown(void) { return NVML_SUCCESS; }

nvmlReturn_t nvmlDeviceGetHandleByIndex_v2(unsigned int i, nvmlDevice_t *d) {
    if (i >= 8) return NVML_ERROR_INVALID_ARGUMENT;
    *d = (nvmlDevice_t)(uintptr_t)(i + 1);
    return NVML_SUCCESS;
}

nvmlReturn_t nvmlDeviceGetPowerUsage(nvmlDevice_t d, unsigned int *mw) {
    *mw = (unsigned int)(watts_at(dev_of(d), now_us()) * 1000.0);
    return NVML_SUCCESS;
}

nvmlReturn_t nvmlDeviceGetFieldValues(nvmlDevice_t d, int n, nvmlFieldValue_t *v) {
    for (int i = 0; i < n; ++i) {
        if (v[i].fieldId == NVML_FI_DEV_POWER_INSTANT) {
            v[i].nvmlReturn = NVML_SUCCESS;
            v[i].valueType = NVML_VALUE_TYPE_UNSIGNED_INT;
            v[i].value.uiVal = (unsigned int)((watts_at(dev_of(d), now_us()) + 50.0) * 1000.0);
        } else {
            v[i].nvmlReturn = NVML_ERROR_NOT_SUPPORTED;
        }
    }
    return NVML_SUCCESS;
}

nvmlReturn_t nvmlDeviceGetSamples(nvmlDevice_t d, nvmlSamplingType_t type, unsigned long long last,
                                  nvmlValueType_t *vt, unsigned int *count, nvmlSample_t *samples) {
    if (type != NVML_TOTAL_POWER_SAMPLES) return NVML_ERROR_NOT_SUPPORTED;
    const int64_t step = 20000, now = now_us();
    int64_t first = ((int64_t)last / step + 1) * step;
    if (first < now - 2000000) first = (now - 2000000) / step * step;  /* the buffer holds 2 s */
    unsigned int n = first <= now ? (unsigned int)((now - first) / step + 1) : 0;
    *vt = NVML_VALUE_TYPE_UNSIGNED_INT;
    if (!samples) {
        *count = n;
        return NVML_SUCCESS;
    }
    if (n > *count) n = *count;
    for (unsigned int i = 0; i < n; ++i) {
        const int64_t t = first + (int64_t)i * step;
        samples[i].timeStamp = (unsigned long long)t;
        samples[i].sampleValue.uiVal = (unsigned int)(watts_at(dev_of(d), t) * 1000.0);
    }
    *count = n;
    return NVML_SUCCESS;
}
