/* summary_harness.c - drives a rung-summary emitter (gpl_summary_emit) on
 * CPU with fixed, synthetic telemetry, so two emitters can be compared field
 * by field: the reference's runner/src/summary.c and the drop-in
 * gpu-power-lab_b200/runner/summary.c. TEST INFRASTRUCTURE, built by
 * tests/test_summary_emitter.py.
 *
 * NVML is replaced by fakes below (no driver is needed), so the device
 * identity comes from fixed strings and the throttle names from a small
 * fixed table.
 *
 * Usage: summary_harness OUT.json OP PREC SIZE ITERS FIXED_WORK DUTY_ON_MS [ERROR_MESSAGE]
 */
#include <nvml.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "args.h"
#include "summary.h"
#include "telemetry.h"
#include "util.h"
#include "workload.h"

/* ---- NVML fakes --------------------------------------------------------- */

static nvmlReturn_t copy_str(char *dst, unsigned int len, const char *s) {
    snprintf(dst, len, "%s", s);
    return NVML_SUCCESS;
}
nvmlReturn_t nvmlDeviceGetUUID(nvmlDevice_t d, char *s, unsigned int n) {
    return copy_str(s, n, "GPU-11111111-2222-3333-4444-555555555555");
}
nvmlReturn_t nvmlDeviceGetName(nvmlDevice_t d, char *s, unsigned int n) { return copy_str(s, n, "NVIDIA B200"); }
nvmlReturn_t nvmlSystemGetDriverVersion(char *s, unsigned int n) { return copy_str(s, n, "580.159"); }
nvmlReturn_t nvmlDeviceGetVbiosVersion(nvmlDevice_t d, char *s, unsigned int n) {
    return copy_str(s, n, "97.00.00.00.01");
}
nvmlReturn_t nvmlDeviceGetPciInfo(nvmlDevice_t d, nvmlPciInfo_t *p) {
    memset(p, 0, sizeof *p);
    snprintf(p->busId, sizeof p->busId, "00000000:1B:00.0");
    return NVML_SUCCESS;
}
nvmlReturn_t nvmlDeviceGetPowerManagementLimit(nvmlDevice_t d, unsigned int *mw) {
    *mw = 1000000;
    return NVML_SUCCESS;
}
nvmlReturn_t nvmlDeviceGetPowerManagementDefaultLimit(nvmlDevice_t d, unsigned int *mw) {
    *mw = 1000000;
    return NVML_SUCCESS;
}
nvmlReturn_t nvmlDeviceGetPowerManagementLimitConstraints(nvmlDevice_t d, unsigned int *lo, unsigned int *hi) {
    *lo = 200000;
    *hi = 1100000;
    return NVML_SUCCESS;
}

/* the kept sampler's name table is not linked; two fixed names stand in */
int gpl_throttle_reason_names(uint64_t mask, const char **out, int max) {
    int n = 0;
    if ((mask & 0x4) && n < max) out[n++] = "sw_power_cap";
    if ((mask & 0x20) && n < max) out[n++] = "sw_thermal_slowdown";
    return n;
}

static gpl_op_t op_of(const char *s) {
    for (int o = GPL_OP_SGEMM; o <= GPL_OP_NCCL; ++o)
        if (!strcmp(gpl_op_name((gpl_op_t)o), s)) return (gpl_op_t)o;
    return GPL_OP_SGEMM;
}

static gpl_prec_t prec_of(const char *s) {
    for (int p = GPL_PREC_FP32; p <= GPL_PREC_FP4; ++p)
        if (!strcmp(gpl_prec_name((gpl_prec_t)p), s)) return (gpl_prec_t)p;
    return GPL_PREC_FP32;
}

static void series(gpl_dvec *v, int n, double base, double step, int period) {
    gpl_dvec_init(v, (size_t)n);
    for (int i = 0; i < n; ++i) gpl_dvec_push(v, base + step * (double)(i % period));
}

int main(int argc, char **argv) {
    if (argc < 8) {
        fprintf(stderr, "usage: %s OUT OP PREC SIZE ITERS FIXED_WORK DUTY_ON_MS [ERROR]\n", argv[0]);
        return 2;
    }
    gpl_args_t a;
    gpl_args_defaults(&a);
    a.op = op_of(argv[2]);
    a.precision = prec_of(argv[3]);
    a.size = atoi(argv[4]);
    a.streams = 1;
    a.warmup_sec = 1.0;
    a.steady_sec = 2.0;
    a.sample_hz = 50;
    a.device = 0;
    a.iters = atoi(argv[6]) ? atoll(argv[5]) : 0;
    a.duty_on_ms = atof(argv[7]);
    a.duty_off_ms = a.duty_on_ms;

    gpl_device_info_t dev;
    gpl_device_info_fill((nvmlDevice_t)0, &dev);

    gpl_telemetry_t tele;
    memset(&tele, 0, sizeof tele);
    gpl_phase_stats_t *s = &tele.steady;
    const int n = 97;
    series(&s->power_w, n, 640.0, 37.5, 11);
    series(&s->power_instant_w, n, 300.0, 71.0, 13);
    series(&s->temp_c, n, 51.0, 0.5, 7);
    series(&s->sm_mhz, n, 1965.0, -45.0, 5);
    series(&s->mem_mhz, n, 3996.0, 0.0, 1);
    series(&s->sm_util, n, 90.0, 2.0, 6);
    series(&s->mem_util, n, 40.0, 5.0, 9);
    s->throttle_mask_or = 0x4;
    s->throttled_sec = 0.75;
    s->energy_start_mj = 123456789ull;
    s->energy_end_mj = 123456789ull + 1617250ull;
    s->energy_valid = true;
    s->samples = (uint64_t)n;
    s->power_integral_j = 1598.125;
    s->elapsed_s = 2.0125;
    s->violation_us_start = 7000000000ull;           /* raw NVML counter values */
    s->violation_us_end = 7000000000ull + 412345678ull;
    s->violation_valid = true;
    s->peak_instant_w = 1187.5;

    gpl_workload_ctx_t w;
    memset(&w, 0, sizeof w);
    w.args = &a;
    w.tele = &tele;
    w.iterations_warmup = 11;
    w.iterations_steady = (uint64_t)atoll(argv[5]);
    w.compute_seconds_steady = 1.9875;

    FILE *f = fopen(argv[1], "w");
    if (!f) return 3;
    const char *err = argc > 8 ? argv[8] : NULL;
    int rc = gpl_summary_emit(f, &a, &dev, &w, &tele, "2026-12-01T12:00:00.000Z", 1000500000ull, 2008660000ull,
                              3084530000ull, NULL, err ? "cuda_error" : "ok", err);
    fclose(f);
    return rc == 0 ? 0 : 4;
}
