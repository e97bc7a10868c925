"""bench.py on the host: the workload table covers every task operator, and the reference arm (the
task's CPU algorithm through the oracle port) prints one JSON line with the contract's keys.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402

TASK_WORKLOADS = {
    "softmax_8192x2048", "reduction_sum_4096x4096", "rope_2x32x1024x128", "silu_16777216", "swiglu_16777216", "gemm_nn_2048",
    "bitdelta_gemm_512x4096x4096", "attention_full_2x8x1024x64", "varlen_kda_h64_mixed", "relu_16777216", "sigmoid_16777216",
    "sigmoid_shift_16777216", "lion_8388608", "gemv_4096x4096", "gemm_silu_2048", "kda_fixed_256x8x64",
}


def test_every_task_operator_has_a_bench_workload():
    assert TASK_WORKLOADS <= set(bench.WORKLOADS)
    assert bench.DEFAULT_WORKLOAD in bench.WORKLOADS


@pytest.mark.parametrize("workload", ["gemv_4096x4096", "kda_fixed_256x8x64"])
def test_reference_arm_prints_the_contract_line(workload):
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", workload, "--steps", "1",
                           "--warmup", "3"], capture_output=True, text=True, cwd=ROOT, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e", "impl"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    assert d["cpu_baseline"]["kind"] in ("port", "reference") and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]


def test_warmup_below_three_is_refused():
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", "gemv_4096x4096",
                           "--steps", "1", "--warmup", "1"], capture_output=True, text=True, cwd=ROOT, timeout=300)
    assert proc.returncode != 0 and "--warmup must be >= 3" in proc.stderr
