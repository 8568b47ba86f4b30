"""Generates the golden fixtures in this directory. Run in a checkout that
has the reference tree and oracle/_ref built (oracle/ref_build.sh):

    python tests/golden/make_golden.py

Fixtures:
  e4m3.json        all 256 E4M3 ("fn") codes decoded by torch.float8_e4m3fn,
                   and torch's encoding of a seeded grid of in-range values
  role_maps.json   the reference's build_role_map (runner/src/
                   workload_powervirus.cu:414-454, compiled from its own
                   source into oracle/_ref/libgpl_ref.so) for a set of mixes
  accounting.json  the reference's gpl_workload_{flops,bytes}_per_iter
                   (runner/src/workload_util.c:20-58) for the ladder sizes
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))
import oracle  # noqa: E402


def e4m3() -> dict:
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn)
    dec = codes.to(torch.float32).numpy()
    rng = np.random.default_rng(20261201)
    # In-range values (|x| <= 448) across the whole exponent range, plus
    # exact ties and subnormals.
    mags = np.concatenate([
        np.exp2(rng.uniform(-11, 8.8, 1200)),
        np.arange(0, 64) * 2.0 ** -10,        # subnormal grid and its midpoints
        np.array([448.0, 447.0, 440.0, 416.0, 432.0, 1.0625, 1.1875, 0.0009765625]),
    ])
    vals = np.concatenate([mags, -mags]).astype(np.float32)
    vals = vals[np.abs(vals) <= 448.0]
    enc = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return {
        "decode": [None if np.isnan(v) else float(v) for v in dec],
        "encode_in": [float(v) for v in vals],
        "encode_out": [int(c) for c in enc],
    }


MIXES = [
    [1, 1, 1, 0, 0, 0, 0, 0],
    [0, 1, 0, 0, 0, 0, 0, 0],
    [5, 1, 1, 1, 0, 0, 0, 0],
    [1, 1, 1, 1, 1, 1, 1, 1],
    [2, 1, 1, 0, 0, 0, 0, 0],
    [0, 0, 0, 0, 0, 0, 0, 0],
    [100, 1, 0, 0, 0, 0, 0, 1],
    [3, 7, 11, 0, 2, 0, 5, 1],
    [1, 0, 0, 0, 0, 0, 0, 0],
    [0, 3, 1, 0, 0, 0, 0, 0],
]


def role_maps() -> list:
    out = []
    for w in MIXES:
        for tc in (False, True):
            m, c = oracle.ref_role_map(w, tensor_cublas=tc)
            out.append({"weights": w, "tensor_cublas": tc, "map": m.tolist(), "counts": c.tolist()})
    return out


def accounting() -> list:
    L = oracle.ref_lib()
    out = []
    for op in ("sgemm", "memstream"):
        for prec in ("fp32", "fp8", "fp4"):
            for size in (256, 1024, 2048, 4096, 8192, 16384, 32768):
                out.append({
                    "op": op, "precision": prec, "size": size,
                    "flops": L.ref_flops_per_iter(oracle.OP[op], oracle.PREC[prec], size),
                    "bytes": L.ref_bytes_per_iter(oracle.OP[op], size),
                })
    return out


def main() -> None:
    (HERE / "e4m3.json").write_text(json.dumps(e4m3()))
    (HERE / "role_maps.json").write_text(json.dumps(role_maps(), indent=0))
    (HERE / "accounting.json").write_text(json.dumps(accounting(), indent=0))
    print("wrote", [p.name for p in HERE.glob("*.json")])


if __name__ == "__main__":
    main()
