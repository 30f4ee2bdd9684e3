"""bench.py's reference arm on the CPU: one JSON line per run with the keys
the measurement contract names, for every workload, and nothing from ranks
other than 0.  (The GPU arm is run on a B200; its line carries the same keys
plus roofline, clocks and launches.)"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
        "cpu_baseline", "e2e"}


def run_bench(*args, env=None):
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", *args],
                       cwd=ROOT, capture_output=True, text=True, timeout=600,
                       env={**os.environ, **(env or {})})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    return lines


@pytest.mark.parametrize("workload,extra,unit", [
    ("dit", ["--cpu-rows", "8"], "TFLOP/s"),
    ("ffn", ["--cpu-rows", "8"], "TFLOP/s"),
    ("quant", ["--cpu-rows", "16"], "GB/s"),
    ("attention", ["--cpu-rows", "16", "--attn-docs", "512,256"], "TFLOP/s"),
    ("refblock", ["--cpu-rows", "8"], "TFLOP/s"),
    ("refblock-shims", ["--cpu-rows", "8"], "TFLOP/s"),
])
def test_reference_arm_line(workload, extra, unit):
    lines = run_bench("--workload", workload, "--steps", "1", "--warmup", "0",
                      "--cpu-seconds", "0.2", *extra)
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["unit"] == unit and d["value"] > 0
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["ms_per_step"] > 0
    assert d["higher_is_better"] is True and d["vs_baseline"] is None
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == unit and cb["cores"] >= 1
    assert cb["kind"] == "port" and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": unit, "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert isinstance(d["config"], dict) and d["config"]["workload"]


def test_reference_arm_other_ranks_print_nothing():
    lines = run_bench("--workload", "quant", "--steps", "1", "--warmup", "0",
                      "--cpu-seconds", "0.1", "--cpu-rows", "8", env={"RANK": "1"})
    assert lines == []
