"""Sustained power of the powervirus and tensor rungs, reference runner
against the drop-in runner, on the same box (run on a GPU; not collected by
pytest):

    python tests/perf_power_rungs.py [--steady 10] [--warmup 3]

Both binaries come from oracle/runner_build.sh. Each rung is one runner
process with the reference's CLI; its summary JSON gives the NVML-sampled
average and peak power and the percentage of the enforced power limit.
No power-limit or clock flag is passed: the GPU's settings are left alone.
Prints one JSON object with a row per rung.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import tempfile
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
REF = REPO / "oracle/_ref/gpu-power-runner"
GPLK = REPO / "oracle/_ref/gpu-power-runner-gplk"

RUNGS = [
    # (label, binary, args, extra environment)
    ("ref idle (observe)", REF, ["--op", "observe"], {}),
    ("ref cuBLASLt fp8 tensor-only 8192", REF, ["--op", "powervirus", "--tensor-backend", "cublas", "--precision",
                                                "fp8", "--size", "8192", "--mix-fma", "0", "--mix-dram", "0"], {}),
    ("ref cuBLAS bf16 tensor-only 8192", REF, ["--op", "powervirus", "--tensor-backend", "cublas", "--precision",
                                               "bf16", "--size", "8192", "--mix-fma", "0", "--mix-dram", "0"], {}),
    ("ref wmma mix 1:1:1", REF, ["--op", "powervirus", "--size", "8192"], {}),
    ("gplk tcgen05 fp8 tensor-only 8192", GPLK, ["--op", "powervirus", "--tensor-backend", "cublas", "--precision",
                                                 "fp8", "--size", "8192", "--mix-fma", "0", "--mix-dram", "0"], {}),
    ("gplk tcgen05 bf16 tensor-only 8192", GPLK, ["--op", "powervirus", "--tensor-backend", "cublas", "--precision",
                                                  "bf16", "--size", "8192", "--mix-fma", "0", "--mix-dram", "0"], {}),
    ("gplk tcgen05 int8 tensor-only 8192", GPLK, ["--op", "powervirus", "--tensor-backend", "cublas", "--precision",
                                                  "int8", "--size", "8192", "--mix-fma", "0", "--mix-dram", "0"], {}),
    ("gplk tcgen05 nvfp4 tensor-only 16384", GPLK, ["--op", "powervirus", "--tensor-backend", "cublas",
                                                    "--precision", "fp4", "--size", "16384", "--mix-fma", "0",
                                                    "--mix-dram", "0"], {}),
    ("gplk in-kernel mix 1:1:1", GPLK, ["--op", "powervirus", "--size", "8192"], {}),
    ("gplk in-kernel mix 2:1:1", GPLK, ["--op", "powervirus", "--size", "8192", "--mix-tensor", "2"], {}),
    ("gplk in-kernel mix 2:1:1 budget 1ms", GPLK, ["--op", "powervirus", "--size", "8192", "--mix-tensor", "2"],
     {"GPL_PV_BUDGET_US": "1000"}),
    ("gplk in-kernel mix 4:1:2 budget 1ms", GPLK, ["--op", "powervirus", "--size", "8192", "--mix-tensor", "4",
                                                   "--mix-dram", "2"], {"GPL_PV_BUDGET_US": "1000"}),
    ("gplk in-kernel mix 2:1:1:sfu1 budget 1ms", GPLK, ["--op", "powervirus", "--size", "8192", "--mix-tensor", "2",
                                                        "--mix-sfu", "1"], {"GPL_PV_BUDGET_US": "1000"}),
    ("ref duty 100/100 cuBLASLt fp8", REF, ["--op", "powervirus", "--tensor-backend", "cublas", "--precision", "fp8",
                                            "--size", "8192", "--mix-fma", "0", "--mix-dram", "0",
                                            "--duty-on-ms", "100", "--duty-off-ms", "100"], {}),
    ("gplk duty 100/100 mix 2:1:1 budget 1ms", GPLK, ["--op", "powervirus", "--size", "8192", "--mix-tensor", "2",
                                                      "--duty-on-ms", "100", "--duty-off-ms", "100"],
     {"GPL_PV_BUDGET_US": "1000"}),
]


def run(binary: Path, args: list[str], warmup: float, steady: float, env: dict) -> dict:
    with tempfile.TemporaryDirectory() as td:
        summary = Path(td) / "s.json"
        metrics = Path(td) / "m.ndjson"
        cmd = [str(binary), "--warmup-sec", str(warmup), "--steady-sec", str(steady), "--sample-hz", "100",
               "--out-summary", str(summary), "--out-metrics", str(metrics), *args]
        e = dict(os.environ)
        e.update(env)
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=int(warmup + steady + 120), env=e)
        if not summary.exists():
            return {"error": res.stderr[-500:]}
        s = json.loads(summary.read_text())
        inst = []
        for line in metrics.read_text().splitlines():
            d = json.loads(line)
            if d.get("phase") == "steady" and d.get("power_instant_w", -1) >= 0:
                inst.append(d["power_instant_w"])
        return {
            "result": s["result"],
            "avg_w": s["power"]["avg_w"],
            "p99_w": s["power"]["p99_w"],
            "pct_of_enforced_limit": s["power"]["pct_of_enforced_limit"],
            "enforced_limit_w": s["power"]["enforced_limit_w"],
            "instant_min_w": min(inst) if inst else None,
            "instant_max_w": max(inst) if inst else None,
            "sm_avg_mhz": s["clocks"]["sm_avg_mhz"],
            "throttle": s["throttle"]["reasons"],
            "tflops": s["compute"]["tflops_measured"],
            "iterations": s["compute"]["iterations"],
        }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steady", type=float, default=10.0)
    ap.add_argument("--warmup", type=float, default=3.0)
    ap.add_argument("--only", default="", help="run only rungs whose label contains this text (comma-separated)")
    args = ap.parse_args()
    keep = [k for k in args.only.split(",") if k]
    out = {}
    for label, binary, rung_args, env in RUNGS:
        if keep and not any(k in label for k in keep):
            continue
        out[label] = run(binary, rung_args, args.warmup, args.steady, env)
        print(label, json.dumps(out[label]), flush=True)
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
