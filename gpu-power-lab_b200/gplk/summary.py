"""The rung-summary JSON contract, in two strengths.

The runner's summary emitter (runner/src/summary.c:181-306) writes one JSON
document per rung. gpu-power-lab's consumers check it against
schema/rung-summary.schema.json with a Draft 2020-12 validator
(orchestrator/schema_validate.py:34-63). That version-1 contract closes the
top level (additionalProperties false) and limits `op` to sgemm / fft /
memstream and `precision` to fp32 / tf32 / fp16 / bf16 / fp8, so the
emitter's own `efficiency` and `transient` blocks, and every powervirus,
observe or nccl rung and every fp4 rung, fall outside it.

This module keeps both contracts:

  extended  runner/rung-summary.schema.v1x.json: version 1 plus the ops,
            precisions and blocks the emitter actually writes. A superset:
            whatever passes `strict` passes here.
  strict    the version-1 contract, derived from the extended schema by
            narrowing the enums and dropping the two added blocks, so one
            file is maintained and the two cannot drift.

`to_v1` turns an emitted summary into a strict-valid one where that is
possible (an sgemm / fft / memstream rung at a version-1 precision) and
refuses otherwise, so a consumer that only accepts version 1 never receives
a rung it would misread.
"""
from __future__ import annotations

import copy
import json
from functools import lru_cache
from pathlib import Path

import jsonschema

SCHEMA_PATH = Path(__file__).resolve().parent.parent / "runner" / "rung-summary.schema.v1x.json"

V1_OPS = ("sgemm", "fft", "memstream")
V1_PRECISIONS = ("fp32", "tf32", "fp16", "bf16", "fp8")
EXTENDED_BLOCKS = ("efficiency", "transient")


@lru_cache(maxsize=None)
def _schema_text() -> str:
    return SCHEMA_PATH.read_text(encoding="utf-8")


def load_schema(strict: bool = False) -> dict:
    """The extended schema, or (strict=True) the version-1 contract."""
    schema = json.loads(_schema_text())
    if strict:
        schema["title"] = "Rung summary, version 1"
        inv = schema["properties"]["invocation"]["properties"]
        inv["op"]["enum"] = list(V1_OPS)
        inv["precision"]["enum"] = list(V1_PRECISIONS)
        for block in EXTENDED_BLOCKS:
            schema["properties"].pop(block)
    return schema


def validate_doc(doc: dict, strict: bool = False, where: str = "<document>") -> None:
    """Raise jsonschema.ValidationError naming the first failing path (in
    path order) and how many more errors there are, as
    orchestrator/schema_validate.py:54-63 does."""
    validator = jsonschema.Draft202012Validator(load_schema(strict))
    errors = sorted(validator.iter_errors(doc), key=lambda e: [str(p) for p in e.absolute_path])
    if not errors:
        return
    first = errors[0]
    path_str = " → ".join(str(p) for p in first.absolute_path) or "<root>"
    more = len(errors) - 1
    extra = f" (and {more} more error{'s' if more > 1 else ''})" if more else ""
    raise jsonschema.ValidationError(f"Summary {where} failed validation at [{path_str}]: {first.message}{extra}",
                                     context=first.context)


def validate_summary(path: Path, strict: bool = False) -> None:
    """Validate the summary file at `path`. Raises FileNotFoundError when it
    is missing, json.JSONDecodeError when it is not JSON, and
    jsonschema.ValidationError when it breaks the contract."""
    path = Path(path)
    doc = json.loads(path.read_text(encoding="utf-8"))
    validate_doc(doc, strict=strict, where=str(path))


def to_v1(doc: dict) -> dict:
    """A copy of `doc` that meets the version-1 contract: the efficiency and
    transient blocks are dropped, nothing else changes. Raises ValueError for
    an op or precision version 1 cannot express."""
    inv = doc.get("invocation", {})
    if inv.get("op") not in V1_OPS:
        raise ValueError(f"op {inv.get('op')!r} has no version-1 form (version 1 knows {', '.join(V1_OPS)})")
    if inv.get("precision") not in V1_PRECISIONS:
        raise ValueError(f"precision {inv.get('precision')!r} has no version-1 form "
                         f"(version 1 knows {', '.join(V1_PRECISIONS)})")
    out = copy.deepcopy(doc)
    for block in EXTENDED_BLOCKS:
        out.pop(block, None)
    return out


def main(argv: list[str] | None = None) -> int:
    """python -m gplk.summary [--strict] [--to-v1 OUT] SUMMARY.json
    Exits 0 when valid, 1 when not (the CLI contract of
    orchestrator/schema_validate.py:67-95)."""
    import argparse
    import sys

    ap = argparse.ArgumentParser(description="Validate a rung summary against the rung-summary contract.")
    ap.add_argument("path")
    ap.add_argument("--strict", action="store_true", help="check the version-1 contract instead of the extended one")
    ap.add_argument("--to-v1", metavar="OUT", help="write the version-1 form of the summary to OUT, then check it")
    ns = ap.parse_args(argv)
    target = Path(ns.path)
    if not target.is_file():
        print(f"ERROR: file not found: {target}", file=sys.stderr)
        return 1
    try:
        if ns.to_v1:
            out = to_v1(json.loads(target.read_text(encoding="utf-8")))
            Path(ns.to_v1).write_text(json.dumps(out, indent=2) + "\n", encoding="utf-8")
            validate_summary(Path(ns.to_v1), strict=True)
        else:
            validate_summary(target, strict=ns.strict)
    except (jsonschema.ValidationError, json.JSONDecodeError, ValueError) as e:
        print(f"INVALID: {e}", file=sys.stderr)
        return 1
    print(f"OK: {target}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
