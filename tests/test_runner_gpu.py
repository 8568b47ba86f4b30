"""The drop-in load generators inside the reference's own runner host.

oracle/runner_build.sh links the reference's kept host (CLI, NVML sampler,
summary emitter, probe, fft/observe/nccl rungs) with this repository's
drop-in workload drivers and libgplk (oracle/_ref/gpu-power-runner-gplk),
and builds the unmodified reference runner beside it
(oracle/_ref/gpu-power-runner). These tests run rungs end to end through
the runner's CLI contract and read its summary JSON and NDJSON telemetry.
No power-limit or clock flag is ever passed: the runners leave the GPU's
settings alone.
"""
from __future__ import annotations

import json
import os
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parent.parent
GPLK_RUNNER = REPO / "oracle/_ref/gpu-power-runner-gplk"
REF_RUNNER = REPO / "oracle/_ref/gpu-power-runner"

needs_runner = pytest.mark.skipif(not GPLK_RUNNER.exists(), reason="runner not built (oracle/runner_build.sh)")


def run_rung(binary: Path, tmp_path: Path, *args: str, env: dict | None = None, timeout: int = 300):
    summary = tmp_path / "summary.json"
    metrics = tmp_path / "metrics.ndjson"
    cmd = [str(binary), "--warmup-sec", "1", "--steady-sec", "2", "--sample-hz", "50",
           "--out-summary", str(summary), "--out-metrics", str(metrics), *args]
    e = dict(os.environ)
    e.update(env or {})
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=e)
    s = json.loads(summary.read_text()) if summary.exists() else None
    lines = metrics.read_text().splitlines() if metrics.exists() else []
    return res, s, lines


def _ok(res, s):
    assert res.returncode == 0, res.stderr[-2000:]
    assert s is not None and s["result"] == "ok", (s or {}).get("error_message")


@needs_runner
def test_memstream_rung(tmp_path):
    res, s, lines = run_rung(GPLK_RUNNER, tmp_path, "--op", "memstream", "--size", "32768",
                             env={"GPL_TRIAD_SCALAR": "3.0"})
    _ok(res, s)
    assert s["invocation"]["op"] == "memstream"
    assert s["throughput"]["op_specific_unit"] == "GB/s"
    assert s["throughput"]["value"] > 5000.0
    assert s["compute"]["iterations"] > 100
    phases = {json.loads(l).get("phase") for l in lines}
    assert "steady" in phases or 2 in phases or "STEADY" in phases


@needs_runner
@pytest.mark.parametrize("prec,size,min_tflops", [("fp32", 1024, 10.0), ("fp8", 8192, 1000.0),
                                                  ("fp4", 8192, 1000.0), ("bf16", 8192, 500.0),
                                                  ("fp16", 8192, 500.0), ("tf32", 8192, 250.0),
                                                  ("int8", 8192, 1000.0), ("fp64", 2048, 1.0)])
def test_gemm_ladder_rungs(prec, size, min_tflops, tmp_path):
    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", "sgemm", "--precision", prec, "--size", str(size))
    _ok(res, s)
    assert s["compute"]["tflops_measured"] > min_tflops, s["compute"]


@needs_runner
@pytest.mark.skipif(not REF_RUNNER.exists(), reason="reference runner not built")
def test_reference_runner_rejects_fp4_on_sgemm(tmp_path):
    """The reference cannot run the NVFP4 rung at all (runner/src/workload_gemm.c:84-89
    rejects fp8/fp4 on this op); the drop-in runs it (test above)."""
    res, s, _ = run_rung(REF_RUNNER, tmp_path, "--op", "sgemm", "--precision", "fp4", "--size", "4096")
    assert res.returncode == 5
    assert s is not None and s["result"] == "cuda_error"


@needs_runner
def test_powervirus_default_mix(tmp_path):
    res, s, lines = run_rung(GPLK_RUNNER, tmp_path, "--op", "powervirus", "--size", "8192")
    _ok(res, s)
    assert s["compute"]["iterations"] > 0
    assert s["power"]["avg_w"] > 0 and s["power"]["pct_of_enforced_limit"] > 0
    assert len(lines) > 10


@needs_runner
@pytest.mark.parametrize("prec,min_tflops", [("fp8", 1000.0), ("fp4", 1000.0), ("bf16", 700.0), ("int8", 1000.0),
                                             ("fp16", 700.0), ("tf32", 350.0), ("fp32", 20.0), ("fp64", 1.0)])
def test_powervirus_tensor_stream(prec, min_tflops, tmp_path):
    """--tensor-backend cublas: GEMMs on a concurrent stream, tensor-only (so
    FLOPs are counted): gpl_lt_* for fp8/fp4, the tcgen05 NN kernels with
    beta = 1 for bf16/fp16/tf32/int8, the SIMT SGEMM with beta = 1 for fp32,
    cublasGemmEx with beta = 1 for fp64."""
    size = "8192" if prec not in ("fp32", "fp64") else "2048"
    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", "powervirus", "--tensor-backend", "cublas",
                         "--precision", prec, "--size", size, "--mix-fma", "0", "--mix-dram", "0")
    _ok(res, s)
    assert s["compute"]["tflops_measured"] > min_tflops


@needs_runner
def test_powervirus_duty_cycle_and_ramp(tmp_path):
    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", "powervirus", "--size", "4096", "--duty-on-ms", "100",
                         "--duty-off-ms", "100", "--duty-ramp", "linear")
    _ok(res, s)
    assert s["transient"]["duty_on_ms"] == 100.0


@needs_runner
def test_powervirus_fixed_work(tmp_path):
    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", "powervirus", "--size", "1024", "--iters", "64",
                         "--mix-tensor", "1", "--mix-fma", "2", "--mix-dram", "1", "--mix-sfu", "1",
                         "--mix-int32", "1", "--mix-smem", "1", "--mix-l2", "1", "--mix-atomic", "1")
    _ok(res, s)
    assert s["compute"]["iterations"] >= 64
    assert s["efficiency"]["mode"] == "fixed_work"


@needs_runner
@pytest.mark.skipif(not REF_RUNNER.exists(), reason="reference runner not built")
def test_memstream_beats_reference_runner(tmp_path):
    """Same rung, same flags, same box: the drop-in's GB/s against the
    reference runner's stream_triad_kernel."""
    (tmp_path / "a").mkdir()
    (tmp_path / "b").mkdir()
    res_r, s_r, _ = run_rung(REF_RUNNER, tmp_path / "a", "--op", "memstream", "--size", "32768")
    _ok(res_r, s_r)
    res_g, s_g, _ = run_rung(GPLK_RUNNER, tmp_path / "b", "--op", "memstream", "--size", "32768")
    _ok(res_g, s_g)
    print(f"memstream GB/s: reference {s_r['throughput']['value']:.0f}, drop-in {s_g['throughput']['value']:.0f}")
    assert s_g["throughput"]["value"] > s_r["throughput"]["value"]


@needs_runner
@pytest.mark.parametrize("op", ["memstream", "sgemm", "powervirus"])
def test_injected_alloc_failure_maps_to_oom(op, tmp_path):
    """Host-side fault injection (GPL_FAULT=alloc): the runner reports result
    "oom" and exits 5, with no GPU fault involved."""
    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", op, "--size", "1024", env={"GPL_FAULT": "alloc"})
    assert res.returncode == 5
    assert s["result"] == "oom" and "injected" in s.get("error_message", "")


@needs_runner
@pytest.mark.parametrize("op", ["memstream", "sgemm", "powervirus"])
def test_injected_launch_failure_maps_to_cuda_error(op, tmp_path):
    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", op, "--size", "1024", env={"GPL_FAULT": "launch"})
    assert res.returncode == 5
    assert s["result"] == "cuda_error" and "injected" in s.get("error_message", "")


@needs_runner
@pytest.mark.parametrize("op,prec,size", [("memstream", "fp32", "32768"), ("sgemm", "fp32", "1024"),
                                          ("sgemm", "fp8", "8192")])
def test_strict_summary_meets_version1_contract(op, prec, size, tmp_path):
    """GPL_SUMMARY_SCHEMA=strict: the drop-in emitter writes the version-1
    document (no efficiency / transient blocks) for rungs version 1 can name."""
    from gplk import summary as S

    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", op, "--precision", prec, "--size", size,
                         env={"GPL_SUMMARY_SCHEMA": "strict"})
    _ok(res, s)
    S.validate_doc(s, strict=True)
    assert "efficiency" not in s and "transient" not in s


@needs_runner
def test_powervirus_summary_extended_contract_and_violation_units(tmp_path):
    """The default summary meets the extended contract, and the power-cap
    violation time is microseconds: never longer than the steady window."""
    from gplk import summary as S

    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", "powervirus", "--size", "4096", "--duty-on-ms", "100",
                         "--duty-off-ms", "100")
    _ok(res, s)
    S.validate_doc(s)
    assert s["transient"]["power_violation_us"] <= s["timing"]["steady_ms"] * 1e3 * 1.05


@needs_runner
def test_tc_gemm_rejects_unaligned_size_with_hint(tmp_path):
    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", "sgemm", "--precision", "int8", "--size", "1000")
    assert res.returncode == 5
    assert s["result"] == "cuda_error" and "multiple of" in s.get("error_message", "")


@needs_runner
@pytest.mark.parametrize("impl", ["gplk", "nccl"])
def test_powervirus_fabric_step_single_rank(impl, tmp_path):
    """The duty cycle with its per-cycle BF16 allreduce (GPL_FABRIC) on one
    rank: every cycle ends with the step, the summary's transient block
    reports it, and the extended schema accepts the document."""
    from gplk import summary as S

    d = tmp_path / "rdv"
    d.mkdir()
    env = {"GPL_FABRIC": impl, "GPL_FABRIC_WORLD": "1", "GPL_FABRIC_RANK": "0", "GPL_FABRIC_DIR": str(d),
           "GPL_FABRIC_MIB": "64", "GPL_PV_BUDGET_US": "1000"}
    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", "powervirus", "--size", "4096", "--mix-tensor", "2",
                         "--duty-on-ms", "100", "--duty-off-ms", "100", env=env)
    _ok(res, s)
    f = s["transient"]["fabric"]
    assert f["impl"] == impl and f["world"] == 1 and f["rank"] == 0 and f["bytes"] == 64 << 20
    assert f["cycles"] == 10  # 2 s steady / 200 ms period
    assert 0.0 < f["median_ms"] <= f["max_ms"] < 100.0
    S.validate_doc(s)


@needs_runner
def test_powervirus_fabric_step_rejects_fixed_work(tmp_path):
    d = tmp_path / "rdv"
    d.mkdir()
    env = {"GPL_FABRIC": "gplk", "GPL_FABRIC_WORLD": "1", "GPL_FABRIC_RANK": "0", "GPL_FABRIC_DIR": str(d)}
    res, s, _ = run_rung(GPLK_RUNNER, tmp_path, "--op", "powervirus", "--size", "1024", "--iters", "8",
                         "--duty-on-ms", "100", "--duty-off-ms", "100", env=env)
    assert res.returncode == 5
    assert s["result"] == "cuda_error" and "fixed work" in s.get("error_message", "")


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


@needs_runner
@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("impl", ["gplk", "nccl"])
def test_powervirus_fabric_step_two_ranks(impl, tmp_path):
    """Two runner processes, one per GPU, in phase: the same number of
    cycles on both, each cycle ending in the 2-rank allreduce."""
    d = tmp_path / "rdv"
    d.mkdir()
    procs, outs = [], []
    for r in range(2):
        out = tmp_path / f"r{r}"
        out.mkdir()
        env = dict(os.environ, GPL_FABRIC=impl, GPL_FABRIC_WORLD="2", GPL_FABRIC_RANK=str(r), GPL_FABRIC_DIR=str(d),
                   GPL_FABRIC_MIB="256", GPL_PV_BUDGET_US="1000", NCCL_NVLS_ENABLE="0")
        cmd = [str(GPLK_RUNNER), "--warmup-sec", "1", "--steady-sec", "2", "--sample-hz", "50", "--device", str(r),
               "--out-summary", str(out / "summary.json"), "--out-metrics", str(out / "metrics.ndjson"),
               "--op", "powervirus", "--size", "4096", "--mix-tensor", "2", "--duty-on-ms", "100",
               "--duty-off-ms", "100"]
        procs.append(subprocess.Popen(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
        outs.append(out)
    for p in procs:
        _, err = p.communicate(timeout=300)
        assert p.returncode == 0, err[-2000:]
    sums = [json.loads((o / "summary.json").read_text()) for o in outs]
    fs = [s["transient"]["fabric"] for s in sums]
    assert [f["rank"] for f in fs] == [0, 1] and all(f["world"] == 2 for f in fs)
    assert fs[0]["cycles"] == fs[1]["cycles"] == 10
    assert all(f["busbw_gbs"] > 50.0 for f in fs)
