"""On the B200: the eval-v2 path end to end (a naive candidate on the gemm_nt task directory, through
the supervised worker) and the calibration probes on a small buffer."""

from __future__ import annotations

import json
from pathlib import Path

import pytest

from shapeforge_b200 import calibrate, eval_task

ROOT = Path(__file__).resolve().parents[1]

NAIVE_GEMM_NT = r'''#include <cuda_fp16.h>
extern "C" __global__ void gemm_nt(const __half* A, const __half* B, __half* C, long long M, long long N, long long K) {
    long long col = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long row = blockIdx.y;
    if (row >= M || col >= N) return;
    float acc = 0.0f;
    for (long long k = 0; k < K; ++k) acc += __half2float(A[row * K + k]) * __half2float(B[col * K + k]);
    C[row * N + col] = __float2half(acc);
}
/* taic-launch
kernel gemm_nt grid=ceil_div(N,128),M threads=128
*/
'''


@pytest.mark.gpu
def test_eval_task_runs_a_candidate_end_to_end(tmp_path, capsys, cuda_device):
    kernel = tmp_path / "gemm_nt.cu"
    kernel.write_text(NAIVE_GEMM_NT)
    rc = eval_task.main([str(ROOT / "tasks" / "gemm_nt"), str(kernel), "--size", "small", "--cases", "normal", "uniform",
                         "--timeout", "300"])
    rep = json.loads(capsys.readouterr().out)
    assert rc == 0 and rep["status"] == "ok", rep
    assert len(rep["cases"]) == 2
    assert rep["pipeline"]["kernel"] == "gemm_nt" and rep["pipeline"]["resident_ctas_per_sm"] >= 1
    bad = tmp_path / "bad.cu"
    bad.write_text(NAIVE_GEMM_NT.replace("acc += ", "acc -= "))
    rc = eval_task.main([str(ROOT / "tasks" / "gemm_nt"), str(bad), "--size", "small", "--cases", "normal", "--in-process"])
    assert rc == 1 and json.loads(capsys.readouterr().out)["status"] == "incorrect"


@pytest.mark.gpu
def test_calibration_probes_measure_plausible_peaks(cuda_device):
    bw = calibrate.measure_peak_bandwidth(nbytes=256 * 2**20, iters=5)
    assert 1000.0 < bw["copy4_gbps"] < 10000.0 and 1000.0 < bw["read4_gbps"] < 10000.0, bw
    fl = calibrate.measure_peak_flops(n=2048, iters=3)
    assert 100.0 < fl["fp16"] < 3000.0 and 100.0 < fl["bf16"] < 3000.0, fl
