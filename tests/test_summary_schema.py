"""The rung-summary contract (gplk.summary): the version-1 contract the
reference's consumers check (schema/rung-summary.schema.json, exercised by
orchestrator/tests/test_schema.py), the extended contract the summary
emitter actually meets, and the converter between them.

Runs on CPU. The fixtures under tests/golden/summaries/ are real runner
output captured on a B200 by tests/golden/capture_runner_summaries.sh.
"""
from __future__ import annotations

import copy
import json
import subprocess
import sys
from pathlib import Path

import jsonschema
import pytest

from gplk import summary as S

GOLDEN = Path(__file__).resolve().parent / "golden" / "summaries"
from conftest import reference_root

_REF = reference_root()
REF_SCHEMA = (_REF / "schema" / "rung-summary.schema.json") if _REF else Path("/nonexistent")


def _doc() -> dict:
    """A version-1 summary with the fields in the emitter's order
    (runner/src/summary.c:181-306), minus the two extended blocks."""
    return {
        "schema_version": 1,
        "rung_id": "b200-0001-memstream-fp32-32768-s1",
        "invocation": {"op": "memstream", "precision": "fp32", "size": 32768, "streams": 1,
                       "warmup_sec": 1.0, "steady_sec": 2.0, "sample_hz": 50, "device": 0},
        "device": {"uuid": "GPU-00000000-0000-0000-0000-000000000000", "name": "NVIDIA B200",
                   "driver": "580.159", "cuda_runtime": "12.9", "vbios": "97.00.00.00.00",
                   "pci_bus_id": "00000000:00:00.0", "power_limit_w": 1000.0},
        "timing": {"start_utc": "2026-12-01T12:00:00.000Z", "warmup_ms": 1000.5, "steady_ms": 2000.25,
                   "wall_ms": 3400.0},
        "compute": {"iterations": 5000, "tflops_measured": 0.0, "tflops_theoretical": None, "efficiency": None},
        "power": {"avg_w": 820.5, "peak_w": 901.0, "p50_w": 818.0, "p95_w": 880.0, "p99_w": 899.0,
                  "energy_j": 1641.0},
        "thermal": {"avg_c": 55.0, "peak_c": 60.0, "throttled_sec": 0.0},
        "throttle": {"mask": 0, "any_throttled": False, "reasons": []},
        "utilization": {"sm_avg_pct": 100.0, "mem_avg_pct": 97.5},
        "clocks": {"sm_avg_mhz": 1965.0, "sm_min_mhz": 1950.0, "sm_max_mhz": 1965.0, "mem_avg_mhz": 3996.0,
                   "sm_boost_dropped": False},
        "samples_written": 100,
        "result": "ok",
        "throughput": {"op_specific_unit": "GB/s", "value": 7080.0},
    }


def _emitted() -> dict:
    """_doc() with the efficiency and transient blocks the emitter always writes."""
    d = _doc()
    d["efficiency"] = {"mode": "fixed_time", "work_unit": "iteration", "work_done": 5000.0, "delay_s": 2.0,
                       "energy_j": 1641.0, "energy_per_work_j": 0.3282, "delay_per_work_s": 0.0004,
                       "edp_j_s": 0.00013128, "edpp_j_s2": 5.2512e-08, "perf_per_watt": 3.047}
    d["transient"] = {"duty_on_ms": 0.0, "duty_off_ms": 0.0, "power_violation_us": 0, "energy_counter_j": 1641.0,
                      "energy_integrated_j": 1639.2, "energy_gap_pct": 0.11, "sample_hz_requested": 50,
                      "sample_hz_achieved": 49.6}
    return d


def _set(d: dict, keys: list, value) -> dict:
    d = copy.deepcopy(d)
    t = d
    for k in keys[:-1]:
        t = t[k]
    t[keys[-1]] = value
    return d


def _valid(doc, strict):
    try:
        S.validate_doc(doc, strict=strict)
        return True
    except jsonschema.ValidationError:
        return False


BOTH = pytest.mark.parametrize("strict", [False, True], ids=["extended", "strict"])


# --- cases of orchestrator/tests/test_schema.py, under both contracts --------

@BOTH
def test_version1_document_is_valid(strict, tmp_path):
    p = tmp_path / "s.json"
    p.write_text(json.dumps(_doc()))
    S.validate_summary(p, strict=strict)


@BOTH
def test_error_message_and_throttle_hit_are_valid(strict):
    S.validate_doc(_set(_set(_doc(), ["result"], "cuda_error"), ["error_message"], "launch failed"), strict=strict)
    d = _set(_doc(), ["result"], "throttle_hit")
    d = _set(d, ["throttle", "any_throttled"], True)
    d = _set(d, ["throttle", "mask"], 4)
    d = _set(d, ["throttle", "reasons"], ["sw_power_cap"])
    S.validate_doc(_set(d, ["thermal", "throttled_sec"], 1.5), strict=strict)


@BOTH
def test_every_version1_enum_value_is_valid(strict):
    for op in S.V1_OPS:
        S.validate_doc(_set(_doc(), ["invocation", "op"], op), strict=strict)
    for prec in S.V1_PRECISIONS:
        S.validate_doc(_set(_doc(), ["invocation", "precision"], prec), strict=strict)
    for r in ("ok", "throttle_hit", "oom", "cuda_error", "nvml_error", "aborted"):
        S.validate_doc(_set(_doc(), ["result"], r), strict=strict)


def _drop(keys):
    def f(d):
        d = copy.deepcopy(d)
        t = d
        for k in keys[:-1]:
            t = t[k]
        del t[keys[-1]]
        return d
    return f


INVALID = {
    "missing_schema_version": _drop(["schema_version"]),
    "schema_version_2": lambda d: _set(d, ["schema_version"], 2),
    "missing_rung_id": _drop(["rung_id"]),
    "empty_rung_id": lambda d: _set(d, ["rung_id"], ""),
    "unknown_op": lambda d: _set(d, ["invocation", "op"], "unknown_op"),
    "unknown_precision": lambda d: _set(d, ["invocation", "precision"], "fp128"),
    "negative_avg_w": lambda d: _set(d, ["power", "avg_w"], -1.0),
    "missing_p50_w": _drop(["power", "p50_w"]),
    "extra_top_level": lambda d: _set(d, ["unexpected_field"], "x"),
    "bad_result": lambda d: _set(d, ["result"], "great_success"),
    "sm_util_over_100": lambda d: _set(d, ["utilization", "sm_avg_pct"], 101.0),
    "steady_below_1s": lambda d: _set(d, ["invocation", "steady_sec"], 0.5),
    "streams_over_64": lambda d: _set(d, ["invocation", "streams"], 65),
    "throughput_extra_key": lambda d: _set(d, ["throughput", "note"], "x"),
    "throughput_bad_unit": lambda d: _set(d, ["throughput", "op_specific_unit"], "MB/s"),
    "efficiency_ratio_over_2": lambda d: _set(d, ["compute", "efficiency"], 2.5),
}


@BOTH
@pytest.mark.parametrize("case", sorted(INVALID))
def test_invalid_documents_are_rejected(case, strict):
    with pytest.raises(jsonschema.ValidationError):
        S.validate_doc(INVALID[case](_doc()), strict=strict)


def test_missing_file_raises(tmp_path):
    with pytest.raises(FileNotFoundError):
        S.validate_summary(tmp_path / "no_such_file.json")


def test_error_names_first_path_and_count():
    d = _set(_set(_doc(), ["power", "avg_w"], -1.0), ["utilization", "sm_avg_pct"], 101.0)
    with pytest.raises(jsonschema.ValidationError) as ei:
        S.validate_doc(d, where="x.json")
    msg = str(ei.value.message)
    assert msg.startswith("Summary x.json failed validation at [power → avg_w]")
    assert "(and 1 more error)" in msg


# --- what the extension adds ---------------------------------------------------

@pytest.mark.parametrize("op,prec", [("powervirus", "fp32"), ("observe", "fp32"), ("nccl", "bf16"),
                                     ("sgemm", "fp4"), ("sgemm", "int8"), ("sgemm", "fp64")])
def test_extended_ops_and_precisions(op, prec):
    d = _set(_set(_doc(), ["invocation", "op"], op), ["invocation", "precision"], prec)
    assert _valid(d, strict=False)
    assert not _valid(d, strict=True)


def test_emitter_blocks_valid_extended_only():
    assert _valid(_emitted(), strict=False)
    assert not _valid(_emitted(), strict=True)


def test_extended_blocks_are_checked():
    assert not _valid(_set(_emitted(), ["efficiency", "mode"], "sometimes"), strict=False)
    assert not _valid(_drop(["transient", "duty_on_ms"])(_emitted()), strict=False)
    assert not _valid(_set(_emitted(), ["transient", "power_violation_us"], -3), strict=False)


def test_to_v1_drops_only_the_extended_blocks():
    src = _emitted()
    out = S.to_v1(src)
    S.validate_doc(out, strict=True)
    assert "efficiency" in src and "transient" in src  # the input is untouched
    assert out == _doc()


@pytest.mark.parametrize("op,prec", [("powervirus", "fp32"), ("sgemm", "fp4")])
def test_to_v1_refuses_what_version1_cannot_express(op, prec):
    d = _set(_set(_emitted(), ["invocation", "op"], op), ["invocation", "precision"], prec)
    with pytest.raises(ValueError):
        S.to_v1(d)


def test_strict_is_a_narrowing_of_extended():
    ext, strict = S.load_schema(False), S.load_schema(True)
    assert set(strict["properties"]) == set(ext["properties"]) - set(S.EXTENDED_BLOCKS)
    assert strict["required"] == ext["required"]
    jsonschema.Draft202012Validator.check_schema(ext)
    jsonschema.Draft202012Validator.check_schema(strict)


def test_cli(tmp_path):
    src = tmp_path / "in.json"
    src.write_text(json.dumps(_emitted()))
    pkg = Path(S.__file__).resolve().parent.parent
    run = lambda *a: subprocess.run([sys.executable, "-m", "gplk.summary", *a], cwd=pkg, capture_output=True,
                                    text=True)
    assert run(str(src)).returncode == 0
    assert run("--strict", str(src)).returncode == 1
    out = tmp_path / "v1.json"
    assert run("--to-v1", str(out), str(src)).returncode == 0
    S.validate_summary(out, strict=True)
    assert run(str(tmp_path / "missing.json")).returncode == 1


# --- the strict contract is the reference's, case by case --------------------

@pytest.mark.skipif(not REF_SCHEMA.exists(), reason="reference schema not present")
def test_strict_matches_reference_schema_on_every_case():
    ref = jsonschema.Draft202012Validator(json.loads(REF_SCHEMA.read_text()))
    docs = [_doc(), _emitted()] + [f(_doc()) for f in INVALID.values()] + [f(_emitted()) for f in INVALID.values()]
    for op in ("sgemm", "fft", "memstream", "powervirus", "observe", "nccl"):
        for prec in ("fp32", "tf32", "fp16", "bf16", "fp8", "fp64", "int8", "fp4"):
            docs.append(_set(_set(_doc(), ["invocation", "op"], op), ["invocation", "precision"], prec))
    docs += [json.loads(p.read_text()) for p in sorted(GOLDEN.glob("*.json"))]
    for d in docs:
        assert ref.is_valid(d) == _valid(d, strict=True), json.dumps(d.get("invocation"))


# --- real runner output --------------------------------------------------------

def _fixtures():
    return sorted(GOLDEN.glob("*.json"))


def test_fixtures_present():
    names = {p.stem for p in _fixtures()}
    assert {"gplk_memstream", "gplk_sgemm_fp32", "gplk_sgemm_fp8", "gplk_sgemm_fp4", "gplk_powervirus"} <= names


@pytest.mark.parametrize("path", _fixtures(), ids=lambda p: p.stem)
def test_runner_output_meets_extended_contract(path):
    S.validate_summary(path)
    doc = json.loads(path.read_text())
    # The emitter always writes the two extended blocks, so its raw output
    # never meets version 1 ...
    assert "efficiency" in doc and "transient" in doc
    assert not _valid(doc, strict=True)
    # ... and the converter gives a version-1 document exactly where version 1
    # can express the rung.
    inv = doc["invocation"]
    if inv["op"] in S.V1_OPS and inv["precision"] in S.V1_PRECISIONS:
        S.validate_doc(S.to_v1(doc), strict=True)
    else:
        with pytest.raises(ValueError):
            S.to_v1(doc)


def test_violation_time_units_in_captured_summaries():
    """The reference emitter reports NVML's nanosecond violation counter as
    microseconds: its capped powervirus capture claims more power-cap time
    than the steady window lasted. The drop-in emitter's never does."""
    ref = json.loads((GOLDEN / "ref_powervirus_capped.json").read_text())
    assert ref["transient"]["power_violation_us"] / 1e6 > 100 * ref["timing"]["steady_ms"] / 1e3
    assert ref["transient"]["power_violation_us"] / 1e9 <= 1.05 * ref["timing"]["steady_ms"] / 1e3  # as ns it fits
    for p in GOLDEN.glob("gplk_*.json"):
        d = json.loads(p.read_text())
        assert d["transient"]["power_violation_us"] / 1e6 <= 1.05 * d["timing"]["steady_ms"] / 1e3, p.name
