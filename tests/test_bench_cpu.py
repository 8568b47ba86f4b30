"""bench.py on CPU: the file defines each function once, and the reference
arm (host-only) prints the driver's JSON line with its baseline fields."""
from __future__ import annotations

import ast
import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def test_bench_functions_defined_once():
    tree = ast.parse((REPO / "bench.py").read_text())
    names = [n.name for n in tree.body if isinstance(n, ast.FunctionDef)]
    dup = sorted({n for n in names if names.count(n) > 1})
    assert not dup, dup


def test_reference_arm_line():
    res = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=300, cwd=str(REPO))
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["cpu_baseline"]["cores"] >= 1 and line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_reference_arm_other_ranks_print_nothing():
    env = {"RANK": "1", "WORLD_SIZE": "2"}
    import os

    e = dict(os.environ, **env)
    res = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=300, cwd=str(REPO), env=e)
    assert res.returncode == 0 and res.stdout.strip() == ""


def test_host_triad_baseline_reports_one_thread_beside_all_cores():
    sys.path.insert(0, str(REPO))
    import bench

    r = bench.cpu_triad_gbps(0.2, n=1 << 20, threads=2)
    assert r["cores"] == 2 and r["value"] > 0 and r["kind"] == "port"
    assert r["single_thread_gbps"] > 0 and "one thread" in r["single_thread_sample"]
    assert "single_thread_gbps" not in bench.cpu_triad_gbps(0.1, n=1 << 20, threads=2, single=False)
