"""The guarded three-trial correctness runtime and the Backend hooks on the B200.

Safety detection is exercised without faulty kernels: the "violations" are host-side tensor
writes into the runtime's own allocations (a guard byte, an output byte) between the kernel and
the checks, which is exactly what an out-of-bounds or non-deterministic kernel would leave.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops as oref
from shapeforge_b200 import _native, cases, compare, portfolio, protocol, runtime
from shapeforge_b200.backend import CudaBackend

pytestmark = pytest.mark.gpu


def _rmsnorm_setup(rows=64, hidden=512, dtype="fp16"):
    td = cases.TORCH_DTYPE[dtype]
    specs = [runtime.TensorSpec("x", (rows, hidden), td, "input"), runtime.TensorSpec("w", (hidden,), td, "input"),
             runtime.TensorSpec("y", (rows, hidden), td, "output")]
    desc = _native.op_desc("rmsnorm", dtype, dims=(rows, hidden), attrs=(1e-6,))

    def launch(ptrs):
        _native.run_op(desc, ptrs, torch.cuda.current_stream().cuda_stream)

    return specs, launch


def _rmsnorm_case(ci, rows=64, hidden=512, dtype="fp16"):
    case = cases.RMSNORM_CASES[ci]
    inp = cases.rmsnorm_inputs(case, cases.case_seed(0, ci), rows, hidden, dtype)
    ref = oref.rmsnorm(inp["x"].double().numpy(), inp["w"].double().numpy(), 1e-6)
    return case, inp, {"y": ref}, {"y": compare.rms_scale(ref)}


def test_three_trials_pass_for_every_rmsnorm_case(cuda_device):
    specs, launch = _rmsnorm_setup()
    backend = CudaBackend()
    results = backend.run_correctness(cuda_device, launch, specs, [_rmsnorm_case(i) for i in range(6)], rtol=2e-3, atol_rel=1e-3)
    assert len(results) == 6 and all(r.ok for r in results), [r.summary() for r in results]


def test_guard_band_hit_is_a_safety_violation(cuda_device):
    specs, launch = _rmsnorm_setup()
    runner = runtime.CorrectnessRunner(specs, lambda p: None, cuda_device)

    def overflowing(ptrs):
        launch(ptrs)
        buf = runner.buffers["y"]
        buf.raw[runtime.GUARD_BYTES + buf.nbytes + 3] = 0  # one byte past the end of y

    runner.launch = overflowing
    res = runner.run_case(*_rmsnorm_case(0), rtol=2e-3, atol_rel=1e-3)
    assert not res.ok and any("guard" in s for s in res.safety), res.summary()


def test_output_depending_on_initial_contents_is_caught(cuda_device):
    specs, launch = _rmsnorm_setup()
    runner = runtime.CorrectnessRunner(specs, lambda p: None, cuda_device)
    calls = {"n": 0}

    def skips_one_element(ptrs):
        launch(ptrs)
        calls["n"] += 1
        if calls["n"] == 2:  # out2: leave the zero fill in one element, as a kernel that skips it would
            runner.buffers["y"].tensor.view(-1)[5] = 0

    runner.launch = skips_one_element
    res = runner.run_case(*_rmsnorm_case(0), rtol=2e-3, atol_rel=1e-3)
    assert not res.ok and res.nondeterminism, res.summary()


def test_probe_and_candidate_runner(cuda_device):
    b = CudaBackend()
    info = b.probe(cuda_device)
    assert info.matches and info.family == "sm_100" and info.limits["sm_count"] == 148
    specs, launch = _rmsnorm_setup(4096, 4096)
    sets = []
    keep = []
    for s in range(4):
        inp = cases.rmsnorm_bench_inputs(4096, 4096, "fp16", seed=s)
        x, w = inp["x"].to(cuda_device), inp["w"].to(cuda_device)
        y = torch.empty_like(x)
        keep.append((x, w, y))
        sets.append([x.data_ptr(), w.data_ptr(), y.data_ptr()])
    desc = _native.op_desc("rmsnorm", "fp16", dims=(4096, 4096), attrs=(1e-6,))
    cand = b.prepare_bench(desc, sets)
    x0, w0, _ = keep[0]
    base = protocol.cuda_event_runner(lambda i: torch.nn.functional.rms_norm(x0, (4096,), w0, 1e-6))
    noise, stats, attempts = protocol.measure_interleaved({"candidate": cand, "torch_mps": base}, reps=5, kmin=4)
    cand_us = stats["candidate"].median_s * 1e6
    base_us = stats["torch_mps"].median_s * 1e6
    assert 0 < cand_us < 200 and base_us > 0
    meas = portfolio.ShardMeasurement("rmsnorm/4096x4096/benchmark", "benchmark", "candidate", cand_us, base_us)
    rep = portfolio.PerformanceReport.evaluate([meas])
    roof = b.roofline({"min_bytes": 4 * 4096 * 4096 + 2 * 4096, "flops": 4 * 4096 * 4096, "dtype": "fp16"}, cand_us * 1e-6,
                      b.calibration("b200"))
    print(f"rmsnorm 4096^2: candidate {cand_us:.2f} us, torch {base_us:.2f} us, speedup {rep.specialized_hit_speedup}, "
          f"bandwidth fraction {roof['bandwidth_fraction']:.3f}")
    assert roof["bound"] == "memory"
