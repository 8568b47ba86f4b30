"""The drop-in summary emitter (gpu-power-lab_b200/runner/summary.c) against
the reference's (runner/src/summary.c), on CPU.

tests/csrc/summary_harness.c feeds both emitters the same synthetic
telemetry through fake NVML calls. Every field must come out identical,
except the repairs the drop-in makes on purpose:
  * transient.power_violation_us is the reference's value / 1000 (NVML's
    violation counter is in nanoseconds);
  * flop-counted rungs gain throughput {TFLOPS, tflops_measured}.
GPL_SUMMARY_SCHEMA=strict output must meet the version-1 contract.

Builds against the reference's kept host headers and sources (args.c,
util.c, summary.h) where they lie, so it skips when the reference tree is
absent.
"""
from __future__ import annotations

import json
import os
import subprocess
from pathlib import Path

import pytest

from gplk import summary as S

REPO = Path(__file__).resolve().parent.parent
from conftest import reference_root

_REF = reference_root()
REF_SRC = (_REF / "runner" / "src") if _REF else Path("/nonexistent")
DROP = REPO / "gpu-power-lab_b200" / "runner"
CUDA = Path("/usr/local/cuda")

pytestmark = pytest.mark.skipif(not (REF_SRC / "summary.c").exists(), reason="reference runner sources not present")


def _build(out: Path, emitter: Path) -> Path:
    cmd = ["gcc", "-std=gnu11", "-O1", "-Wall", "-Wno-unused-parameter", f"-I{CUDA}/include", f"-I{REF_SRC}",
           str(REPO / "tests/csrc/summary_harness.c"), str(emitter), str(REF_SRC / "args.c"), str(REF_SRC / "util.c"),
           str(DROP / "workload_util.c"), f"-L{CUDA}/lib64", "-lcudart", "-lm", "-o", str(out),
           f"-Wl,-rpath,{CUDA}/lib64"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return out


@pytest.fixture(scope="module")
def harnesses(tmp_path_factory):
    d = tmp_path_factory.mktemp("emit")
    return {"ref": _build(d / "h_ref", REF_SRC / "summary.c"), "drop": _build(d / "h_drop", DROP / "summary.c")}


def _emit(binary: Path, tmp: Path, *args: str, env: dict | None = None):
    out = tmp / f"{binary.name}.json"
    e = dict(os.environ)
    e.pop("GPL_SUMMARY_SCHEMA", None)
    e.update(env or {})
    res = subprocess.run([str(binary), str(out), *args], capture_output=True, text=True, env=e)
    assert res.returncode == 0, res.stderr
    return json.loads(out.read_text()), res.stderr


CASES = [
    ("memstream", "fp32", "32768", "5000", "0", "0"),
    ("sgemm", "fp32", "1024", "4000", "0", "0"),
    ("sgemm", "fp8", "8192", "3000", "1", "0"),
    ("sgemm", "fp4", "16384", "300", "0", "0"),
    ("powervirus", "fp32", "4096", "700", "0", "100"),
    ("fft", "fp32", "4096", "900", "0", "0"),
]


def _flat(d, prefix=""):
    out = {}
    for k, v in d.items():
        if isinstance(v, dict):
            out.update(_flat(v, f"{prefix}{k}."))
        else:
            out[f"{prefix}{k}"] = v
    return out


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{c[1]}")
def test_fields_match_reference_emitter(case, harnesses, tmp_path):
    ref, _ = _emit(harnesses["ref"], tmp_path, *case)
    drop, _ = _emit(harnesses["drop"], tmp_path, *case)
    assert [k for k in drop if k != "throughput" or "throughput" in ref] == list(ref)  # same keys, same order
    fr, fd = _flat(ref), _flat(drop)
    expected_extra = set()
    if drop.get("throughput", {}).get("op_specific_unit") == "TFLOPS":
        assert "throughput" not in ref
        assert drop["throughput"]["value"] == pytest.approx(drop["compute"]["tflops_measured"], rel=1e-6)
        expected_extra = {"throughput.op_specific_unit", "throughput.value"}
    assert set(fd) - set(fr) == expected_extra
    assert set(fr) <= set(fd)
    for k, v in fr.items():
        if k == "transient.power_violation_us":
            assert fd[k] == v // 1000
        else:
            assert fd[k] == v, k


def test_violation_is_microseconds(harnesses, tmp_path):
    drop, _ = _emit(harnesses["drop"], tmp_path, *CASES[4])
    # the harness's counter moved 412 345 678 ns during a 2.0 s steady window
    assert drop["transient"]["power_violation_us"] == 412345
    assert drop["transient"]["power_violation_us"] / 1e6 <= drop["timing"]["steady_ms"] / 1e3


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{c[1]}")
def test_default_output_meets_extended_contract(case, harnesses, tmp_path):
    drop, _ = _emit(harnesses["drop"], tmp_path, *case)
    S.validate_doc(drop)


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{c[1]}")
def test_strict_mode(case, harnesses, tmp_path):
    drop, err = _emit(harnesses["drop"], tmp_path, *case, env={"GPL_SUMMARY_SCHEMA": "strict"})
    op, prec = case[0], case[1]
    if op in S.V1_OPS and prec in S.V1_PRECISIONS:
        S.validate_doc(drop, strict=True)
        assert "efficiency" not in drop and "transient" not in drop
        full, _ = _emit(harnesses["drop"], tmp_path, *case)
        assert S.to_v1(full) == drop
    else:
        assert "no version-1 form" in err
        S.validate_doc(drop)
        assert "efficiency" in drop


def test_strict_output_meets_reference_schema(harnesses, tmp_path):
    ref_schema = (_REF / "schema" / "rung-summary.schema.json") if _REF else None
    if ref_schema is None or not ref_schema.exists():
        pytest.skip("reference schema not present")
    import jsonschema

    v = jsonschema.Draft202012Validator(json.loads(ref_schema.read_text()))
    for case in CASES:
        doc, _ = _emit(harnesses["drop"], tmp_path, *case, env={"GPL_SUMMARY_SCHEMA": "strict"})
        ok = case[0] in S.V1_OPS and case[1] in S.V1_PRECISIONS
        assert v.is_valid(doc) == ok, case
        ref_doc, _ = _emit(harnesses["ref"], tmp_path, *case)
        assert not v.is_valid(ref_doc), "the reference emitter's own output breaks its schema"


def test_error_message_is_escaped(harnesses, tmp_path):
    msg = 'cublasLtMatmul failed: "CUBLAS_STATUS_NOT_SUPPORTED"\tat C:\\path'
    drop, _ = _emit(harnesses["drop"], tmp_path, *CASES[1], msg)
    assert drop["error_message"] == msg and drop["result"] == "cuda_error"
    S.validate_doc(drop)


def test_unknown_schema_mode_falls_back_with_warning(harnesses, tmp_path):
    drop, err = _emit(harnesses["drop"], tmp_path, *CASES[0], env={"GPL_SUMMARY_SCHEMA": "v7"})
    assert "neither 'strict' nor 'extended'" in err
    assert "efficiency" in drop
