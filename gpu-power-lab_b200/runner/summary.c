/* summary.c - the runner's rung-summary emitter, drop-in for
 * runner/src/summary.c (same two entry points, declared by the kept
 * runner/src/summary.h).
 *
 * It writes the document the reference emitter writes, field for field
 * (runner/src/summary.c:181-306), with three repairs:
 *
 *   1. power_violation_us is in microseconds. NVML's violationTime is a
 *      nanosecond counter (nvml.h, nvmlViolationTime_t), and the kept sampler
 *      records its raw value at the first and last steady sample
 *      (runner/src/telemetry.c:196-201), so the steady-window delta it leaves
 *      is in nanoseconds. Dividing by 1000 gives the microseconds the field
 *      name promises; the reference reports the nanosecond delta as is.
 *   2. Every rung whose work is counted in flops (GEMM rungs, tensor-only
 *      powervirus) also gets `throughput` in TFLOPS, the unit the schema
 *      already reserves for it.
 *   3. GPL_SUMMARY_SCHEMA=strict writes the version-1 form: the same document
 *      without the `efficiency` and `transient` blocks, which the version-1
 *      schema's closed top level rejects. Only sgemm / fft / memstream rungs
 *      at fp32 / tf32 / fp16 / bf16 / fp8 have a version-1 form; for any
 *      other rung the extended document is written and a warning is logged.
 *      The default (unset, or GPL_SUMMARY_SCHEMA=extended) is the extended
 *      document, which gpu-power-lab_b200/runner/rung-summary.schema.v1x.json
 *      describes.
 *
 * The extended document's `transient` block also carries `fabric` (the
 * per-cycle allreduce of the multi-GPU powervirus rung: implementation,
 * rank, world, bytes, cycles, median and max time, bus bandwidth) when that
 * step ran; the reference has no such step.
 *
 * Strings are JSON-escaped and non-finite numbers are written as 0, so the
 * output always parses (an error message with a quote in it does not break
 * the document).
 */
#include "summary.h"

#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "fabric_step.h"
#include "util.h"

/* The multi-GPU powervirus rung's per-cycle fabric step reports through
 * gpl_fabric_stats (fabric_step.cu). A weak reference: an emitter linked
 * without that file sees NULL and writes no fabric block. */
#pragma weak gpl_fabric_stats

/* ---- device identity ---------------------------------------------------- */

int gpl_device_info_fill(nvmlDevice_t dev, gpl_device_info_t *out) {
    memset(out, 0, sizeof(*out));
    (void)nvmlDeviceGetUUID(dev, out->uuid, sizeof out->uuid);
    (void)nvmlDeviceGetName(dev, out->name, sizeof out->name);
    (void)nvmlSystemGetDriverVersion(out->driver, sizeof out->driver);
    (void)nvmlDeviceGetVbiosVersion(dev, out->vbios, sizeof out->vbios);

    int rt = 0;
    if (cudaRuntimeGetVersion(&rt) == cudaSuccess)
        snprintf(out->cuda_runtime, sizeof out->cuda_runtime, "%d.%d", rt / 1000, (rt % 1000) / 10);

    nvmlPciInfo_t pci;
    if (nvmlDeviceGetPciInfo(dev, &pci) == NVML_SUCCESS)
        snprintf(out->pci_bus_id, sizeof out->pci_bus_id, "%s", pci.busId);

    unsigned int mw = 0, lo = 0, hi = 0;
    if (nvmlDeviceGetPowerManagementLimit(dev, &mw) == NVML_SUCCESS) out->power_limit_w = mw / 1000.0;
    if (nvmlDeviceGetPowerManagementDefaultLimit(dev, &mw) == NVML_SUCCESS) out->default_limit_w = mw / 1000.0;
    if (nvmlDeviceGetPowerManagementLimitConstraints(dev, &lo, &hi) == NVML_SUCCESS) {
        out->min_limit_w = lo / 1000.0;
        out->max_limit_w = hi / 1000.0;
    }
    return 0;
}

/* ---- a small JSON writer ------------------------------------------------ */

typedef struct {
    FILE *f;
    int depth;
    int count[8]; /* members written so far at each depth */
    int inline_at; /* depth from which objects are written on one line, 0 = never */
} jw_t;

static void jw_sep(jw_t *w, const char *key) {
    int d = w->depth;
    bool inl = w->inline_at && d >= w->inline_at;
    if (w->count[d]++) fputc(',', w->f);
    if (inl) {
        fputc(' ', w->f);
    } else {
        fputc('\n', w->f);
        for (int i = 0; i <= d; i++) fputs("  ", w->f);
    }
    if (key) fprintf(w->f, "\"%s\": ", key);
}

static void jw_str_raw(jw_t *w, const char *s) {
    fputc('"', w->f);
    for (const unsigned char *p = (const unsigned char *)(s ? s : ""); *p; ++p) {
        switch (*p) {
            case '"': fputs("\\\"", w->f); break;
            case '\\': fputs("\\\\", w->f); break;
            case '\n': fputs("\\n", w->f); break;
            case '\r': fputs("\\r", w->f); break;
            case '\t': fputs("\\t", w->f); break;
            default:
                if (*p < 0x20) fprintf(w->f, "\\u%04x", *p);
                else fputc(*p, w->f);
        }
    }
    fputc('"', w->f);
}

static void jw_open(jw_t *w, const char *key, char brace) {
    jw_sep(w, key);
    fputc(brace, w->f);
    w->count[++w->depth] = 0;
}

static void jw_close(jw_t *w, char brace) {
    bool inl = w->inline_at && w->depth >= w->inline_at;
    bool empty = w->count[w->depth] == 0;
    w->depth--;
    if (!empty) {
        if (inl) {
            fputc(' ', w->f);
        } else {
            fputc('\n', w->f);
            for (int i = 0; i <= w->depth; i++) fputs("  ", w->f);
        }
    }
    fputc(brace, w->f);
}

static void jw_num(jw_t *w, const char *key, const char *fmt, double v) {
    jw_sep(w, key);
    fprintf(w->f, fmt, isfinite(v) ? v : 0.0);
}

static void jw_u64(jw_t *w, const char *key, unsigned long long v) {
    jw_sep(w, key);
    fprintf(w->f, "%llu", v);
}

static void jw_int(jw_t *w, const char *key, long long v) {
    jw_sep(w, key);
    fprintf(w->f, "%lld", v);
}

static void jw_bool(jw_t *w, const char *key, bool v) {
    jw_sep(w, key);
    fputs(v ? "true" : "false", w->f);
}

static void jw_null(jw_t *w, const char *key) {
    jw_sep(w, key);
    fputs("null", w->f);
}

static void jw_str(jw_t *w, const char *key, const char *s) {
    jw_sep(w, key);
    jw_str_raw(w, s);
}

/* ---- statistics over a steady-phase series ------------------------------ */

typedef struct {
    double min, max, mean;
} series_t;

static series_t series_of(const gpl_dvec *v) {
    series_t s = {0.0, 0.0, 0.0};
    if (!v->len) return s;
    s.min = s.max = v->data[0];
    double sum = 0.0;
    for (size_t i = 0; i < v->len; ++i) {
        double x = v->data[i];
        s.min = x < s.min ? x : s.min;
        s.max = x > s.max ? x : s.max;
        sum += x;
    }
    s.mean = sum / (double)v->len;
    return s;
}

/* Nearest-rank percentiles of a copy (gpl_dvec_percentile sorts in place). */
static void percentiles(const gpl_dvec *v, double *p50, double *p95, double *p99) {
    *p50 = *p95 = *p99 = 0.0;
    if (!v->len) return;
    gpl_dvec c;
    if (gpl_dvec_init(&c, v->len) != 0) return;
    for (size_t i = 0; i < v->len; ++i) gpl_dvec_push(&c, v->data[i]);
    *p50 = gpl_dvec_percentile(&c, 50.0);
    *p95 = gpl_dvec_percentile(&c, 95.0);
    *p99 = gpl_dvec_percentile(&c, 99.0);
    gpl_dvec_free(&c);
}

static bool version1_expressible(const gpl_args_t *a) {
    bool op = a->op == GPL_OP_SGEMM || a->op == GPL_OP_FFT || a->op == GPL_OP_MEMSTREAM;
    bool prec = a->precision == GPL_PREC_FP32 || a->precision == GPL_PREC_TF32 || a->precision == GPL_PREC_FP16 ||
                a->precision == GPL_PREC_BF16 || a->precision == GPL_PREC_FP8;
    return op && prec;
}

/* GPL_SUMMARY_SCHEMA: "strict" → true, unset / "extended" → false. */
static bool strict_requested(void) {
    const char *e = getenv("GPL_SUMMARY_SCHEMA");
    if (!e || !*e || !strcmp(e, "extended")) return false;
    if (!strcmp(e, "strict")) return true;
    gpl_errf("GPL_SUMMARY_SCHEMA=%s is neither 'strict' nor 'extended'; writing the extended summary", e);
    return false;
}

/* ---- the summary -------------------------------------------------------- */

int gpl_summary_emit(FILE *out, const gpl_args_t *args, const gpl_device_info_t *dev,
                     const gpl_workload_ctx_t *wctx, gpl_telemetry_t *tele, const char *start_utc,
                     uint64_t warmup_ns, uint64_t steady_ns, uint64_t wall_ns, const char *rung_id,
                     const char *result_string, const char *error_message) {
    const gpl_phase_stats_t *st = &tele->steady;
    const double steady_s = (double)steady_ns / 1e9;

    /* power: driver-averaged samples, counter energy where the counter moved */
    const series_t pw = series_of(&st->power_w);
    double p50, p95, p99;
    percentiles(&st->power_w, &p50, &p95, &p99);
    const bool counter_ok = st->energy_valid && st->energy_end_mj >= st->energy_start_mj;
    const double energy_j = counter_ok ? (double)(st->energy_end_mj - st->energy_start_mj) / 1000.0
                                       : pw.mean * steady_s;
    const double tdp_w = dev->default_limit_w > 0.0 ? dev->default_limit_w : dev->power_limit_w;

    const series_t temp = series_of(&st->temp_c);
    const series_t sm = series_of(&st->sm_mhz);
    const series_t mem = series_of(&st->mem_mhz);
    const series_t sm_util = series_of(&st->sm_util);
    const series_t mem_util = series_of(&st->mem_util);

    /* work accounting: flop-bearing rungs count petaflop, others iterations */
    const double iters = (double)wctx->iterations_steady;
    const double busy_s = wctx->compute_seconds_steady;
    const double flops_per_iter = gpl_workload_flops_per_iter(args);
    const bool counted = busy_s > 0.0 && wctx->iterations_steady > 0;
    const double tflops = (flops_per_iter > 0.0 && counted) ? flops_per_iter * iters / busy_s / 1e12 : 0.0;
    const double work = flops_per_iter > 0.0 ? flops_per_iter * iters / 1e15 : iters;
    const double e_per_work = work > 0.0 ? energy_j / work : 0.0;
    const double d_per_work = work > 0.0 ? busy_s / work : 0.0;

    /* transient evidence */
    const double achieved_hz = st->elapsed_s > 0.0 ? (double)st->samples / st->elapsed_s : 0.0;
    const unsigned long long violation_us =
        st->violation_valid && st->violation_us_end >= st->violation_us_start
            ? (unsigned long long)((st->violation_us_end - st->violation_us_start) / 1000u)
            : 0ull;
    const double gap_pct = energy_j > 0.0 ? 100.0 * (energy_j - st->power_integral_j) / energy_j : 0.0;

    char rid[160];
    if (rung_id && *rung_id)
        snprintf(rid, sizeof rid, "%s", rung_id);
    else
        snprintf(rid, sizeof rid, "%s-%s-%d-s%d-%s", gpl_op_name(args->op), gpl_prec_name(args->precision),
                 args->size, args->streams, start_utc);

    bool strict = strict_requested();
    if (strict && !version1_expressible(args)) {
        gpl_errf("GPL_SUMMARY_SCHEMA=strict: a %s %s rung has no version-1 form; writing the extended summary",
                 gpl_op_name(args->op), gpl_prec_name(args->precision));
        strict = false;
    }

    jw_t w = {out, 0, {0}, 2};
    fputc('{', out);
    jw_int(&w, "schema_version", 1);
    jw_str(&w, "rung_id", rid);

    jw_open(&w, "invocation", '{');
    jw_str(&w, "op", gpl_op_name(args->op));
    jw_str(&w, "precision", gpl_prec_name(args->precision));
    jw_int(&w, "size", args->size);
    jw_int(&w, "streams", args->streams);
    jw_num(&w, "warmup_sec", "%.3f", args->warmup_sec);
    jw_num(&w, "steady_sec", "%.3f", args->steady_sec);
    jw_int(&w, "sample_hz", args->sample_hz);
    jw_int(&w, "device", args->device);
    jw_close(&w, '}');

    jw_open(&w, "device", '{');
    jw_str(&w, "uuid", dev->uuid);
    jw_str(&w, "name", dev->name);
    jw_str(&w, "driver", dev->driver);
    jw_str(&w, "cuda_runtime", dev->cuda_runtime);
    jw_str(&w, "vbios", dev->vbios);
    jw_str(&w, "pci_bus_id", dev->pci_bus_id);
    jw_num(&w, "power_limit_w", "%.2f", dev->power_limit_w);
    jw_close(&w, '}');

    jw_open(&w, "timing", '{');
    jw_str(&w, "start_utc", start_utc);
    jw_num(&w, "warmup_ms", "%.2f", (double)warmup_ns / 1e6);
    jw_num(&w, "steady_ms", "%.2f", (double)steady_ns / 1e6);
    jw_num(&w, "wall_ms", "%.2f", (double)wall_ns / 1e6);
    jw_close(&w, '}');

    jw_open(&w, "compute", '{');
    jw_u64(&w, "iterations", (unsigned long long)wctx->iterations_steady);
    jw_num(&w, "tflops_measured", "%.4f", tflops);
    jw_null(&w, "tflops_theoretical");
    jw_null(&w, "efficiency");
    jw_close(&w, '}');

    jw_open(&w, "power", '{');
    jw_num(&w, "avg_w", "%.3f", pw.mean);
    jw_num(&w, "peak_w", "%.3f", pw.max);
    jw_num(&w, "p50_w", "%.3f", p50);
    jw_num(&w, "p95_w", "%.3f", p95);
    jw_num(&w, "p99_w", "%.3f", p99);
    jw_num(&w, "energy_j", "%.3f", energy_j);
    jw_num(&w, "peak_instant_w", "%.3f", st->peak_instant_w);
    jw_str(&w, "sample_source", st->power_instant_w.len ? "nvml_usage+instant" : "nvml_usage");
    jw_num(&w, "tdp_w", "%.2f", tdp_w);
    jw_num(&w, "default_limit_w", "%.2f", dev->default_limit_w);
    jw_num(&w, "enforced_limit_w", "%.2f", dev->power_limit_w);
    jw_num(&w, "max_limit_w", "%.2f", dev->max_limit_w);
    jw_num(&w, "pct_of_tdp", "%.2f", tdp_w > 0.0 ? 100.0 * pw.mean / tdp_w : 0.0);
    jw_num(&w, "pct_of_enforced_limit", "%.2f", dev->power_limit_w > 0.0 ? 100.0 * pw.mean / dev->power_limit_w : 0.0);
    jw_close(&w, '}');

    if (!strict) {
        jw_open(&w, "efficiency", '{');
        jw_str(&w, "mode", args->iters > 0 ? "fixed_work" : "fixed_time");
        jw_str(&w, "work_unit", flops_per_iter > 0.0 ? "pflop" : "iteration");
        jw_num(&w, "work_done", "%.6f", work);
        jw_num(&w, "delay_s", "%.4f", busy_s);
        jw_num(&w, "energy_j", "%.3f", energy_j);
        jw_num(&w, "energy_per_work_j", "%.6f", e_per_work);
        jw_num(&w, "delay_per_work_s", "%.9f", d_per_work);
        jw_num(&w, "edp_j_s", "%.9f", e_per_work * d_per_work);
        jw_num(&w, "edpp_j_s2", "%.12f", e_per_work * d_per_work * d_per_work);
        jw_num(&w, "perf_per_watt", "%.6f", busy_s > 0.0 && pw.mean > 0.0 ? work / busy_s / pw.mean : 0.0);
        jw_close(&w, '}');

        jw_open(&w, "transient", '{');
        jw_num(&w, "duty_on_ms", "%.3f", args->duty_on_ms);
        jw_num(&w, "duty_off_ms", "%.3f", args->duty_off_ms);
        jw_u64(&w, "power_violation_us", violation_us);
        jw_num(&w, "energy_counter_j", "%.3f", energy_j);
        jw_num(&w, "energy_integrated_j", "%.3f", st->power_integral_j);
        jw_num(&w, "energy_gap_pct", "%.3f", gap_pct);
        jw_int(&w, "sample_hz_requested", args->sample_hz);
        jw_num(&w, "sample_hz_achieved", "%.1f", achieved_hz);
        const gpl_fabric_stats_t *fs = gpl_fabric_stats ? gpl_fabric_stats() : NULL;
        if (fs && fs->active) {
            jw_open(&w, "fabric", '{');
            jw_str(&w, "impl", fs->impl);
            jw_int(&w, "rank", fs->rank);
            jw_int(&w, "world", fs->world);
            jw_u64(&w, "bytes", (unsigned long long)fs->bytes);
            jw_u64(&w, "cycles", fs->cycles);
            jw_num(&w, "median_ms", "%.4f", fs->median_ms);
            jw_num(&w, "max_ms", "%.4f", fs->max_ms);
            jw_num(&w, "busbw_gbs", "%.2f", fs->busbw_gbs);
            jw_close(&w, '}');
        }
        jw_close(&w, '}');
    }

    jw_open(&w, "thermal", '{');
    jw_num(&w, "avg_c", "%.2f", temp.mean);
    jw_num(&w, "peak_c", "%.2f", temp.max);
    jw_num(&w, "throttled_sec", "%.3f", st->throttled_sec);
    jw_close(&w, '}');

    const char *names[32];
    const int nnames = gpl_throttle_reason_names(st->throttle_mask_or, names, 32);
    jw_open(&w, "throttle", '{');
    jw_u64(&w, "mask", (unsigned long long)st->throttle_mask_or);
    jw_bool(&w, "any_throttled", st->throttled_sec > 0.0);
    jw_open(&w, "reasons", '[');
    for (int i = 0; i < nnames; ++i) jw_str(&w, NULL, names[i]);
    jw_close(&w, ']');
    jw_close(&w, '}');

    jw_open(&w, "utilization", '{');
    jw_num(&w, "sm_avg_pct", "%.2f", sm_util.mean);
    jw_num(&w, "mem_avg_pct", "%.2f", mem_util.mean);
    jw_close(&w, '}');

    jw_open(&w, "clocks", '{');
    jw_num(&w, "sm_avg_mhz", "%.1f", sm.mean);
    jw_num(&w, "sm_min_mhz", "%.1f", sm.min);
    jw_num(&w, "sm_max_mhz", "%.1f", sm.max);
    jw_num(&w, "mem_avg_mhz", "%.1f", mem.mean);
    jw_bool(&w, "sm_boost_dropped", st->sm_mhz.len > 4 && sm.min < 0.9 * sm.max);
    jw_close(&w, '}');

    jw_u64(&w, "samples_written", (unsigned long long)st->samples);
    jw_str(&w, "result", result_string);
    if (error_message && *error_message) jw_str(&w, "error_message", error_message);

    /* throughput: GB/s for memstream, GFFT/s for fft, TFLOPS for flop-counted rungs */
    if (counted) {
        const double bytes_per_iter = gpl_workload_bytes_per_iter(args);
        const char *unit = NULL;
        double value = 0.0;
        if (args->op == GPL_OP_MEMSTREAM && bytes_per_iter > 0.0) {
            unit = "GB/s";
            value = bytes_per_iter * iters / busy_s / 1e9;
        } else if (args->op == GPL_OP_FFT && bytes_per_iter > 0.0) {
            /* the fft rung's batch: 2^20 points split into transforms of --size */
            int batch = args->size > 0 ? (1 << 20) / args->size : 1;
            unit = "GFFT/s";
            value = (double)(batch < 1 ? 1 : batch) * iters / busy_s / 1e9;
        } else if (tflops > 0.0) {
            unit = "TFLOPS";
            value = tflops;
        }
        if (unit) {
            int saved = w.inline_at;
            w.inline_at = 1;
            jw_open(&w, "throughput", '{');
            jw_str(&w, "op_specific_unit", unit);
            jw_num(&w, "value", "%.4f", value);
            jw_close(&w, '}');
            w.inline_at = saved;
        }
    }
    fputs("\n}\n", out);
    return ferror(out) ? -1 : 0;
}
