"""bench.py's reference arm (CPU): one JSON line per workload with the contract's keys, the same metric, unit and
config workload as the library's arm prints for that workload."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

OUR_METRIC = {
    ("gemm", ()): ("Q4_K dequant-GEMM prefill TFLOP/s", "TFLOP/s", "q4k_prefill_gemm"),
    ("gemv", ("--tokens", "1")): ("Q4_K decode GEMV HBM GB/s (M=1)", "GB/s", "q4k_decode_gemv"),
    ("lmhead", ("--tokens", "1")): ("Q6_K lm-head decode GEMV HBM GB/s (M=1)", "GB/s", "q6k_lm_head_decode_gemv"),
    ("stack", ("--stack-tokens", "64", "--layers", "2")):
        ("Q4_K layer-stack prefill TFLOP/s (tensor-parallel)", "TFLOP/s", "q4k_layer_stack_tp"),
}


@pytest.mark.parametrize("workload,extra", list(OUR_METRIC))
def test_reference_line(workload, extra):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                          workload, "--steps", "1", "--warmup", "3", *extra],
                         capture_output=True, text=True, timeout=600, cwd=ROOT,
                         env={**os.environ, "WORLD_SIZE": "1", "RANK": "0"})
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    metric, unit, name = OUR_METRIC[(workload, extra)]
    assert line["impl"] == "reference"
    assert (line["metric"], line["unit"], line["config"]["workload"]) == (metric, unit, name)
    assert line["value"] > 0 and line["higher_is_better"] is True
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["cores"] >= 1
    assert cb["dequant_ms"] > 0 and cb["gemm_ms"] > 0 and cb["dequant_ms"] + cb["gemm_ms"] <= line["ms_per_step"] * 1.01
    assert line["e2e"] == {"value": line["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_other_ranks_print_nothing():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT,
                         env={**os.environ, "WORLD_SIZE": "2", "RANK": "1"})
    assert out.returncode == 0 and out.stdout.strip() == ""
