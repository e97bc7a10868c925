"""bitdelta_gemm (task contract) and bitdelta_gemm_base (W_base + diag(alpha) S workload) on the B200.

Tolerances: the task's OpSpec ones (tasks/bitdelta_gemm/opspec.json numerics): fp16 rtol 2e-3 /
atol_rel 1e-3, bf16 rtol 1.6e-2 / atol_rel 8e-3, scaled by the RMS of the finite reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle import ops as oref
from shapeforge_b200 import cases, compare, ops
from tests import golden

pytestmark = pytest.mark.gpu

TOL = {"fp16": dict(rtol=2e-3, atol_rel=1e-3), "bf16": dict(rtol=1.6e-2, atol_rel=8e-3)}
TD = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _np(t):
    return t.detach().cpu().to(torch.float64).numpy()


def _status_ok():
    code, where = ops.kernel_status()
    assert code == 0, f"tensor-core kernel status {code} at wait {where}"


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_reference_vectors(cuda_device, dtype):
    """The kernel on the reference module's own inputs (x rows / bit columns sliced) vs its fp64 output."""
    doc = golden.load(f"ref_bitdelta_gemm_{dtype}")
    for rec in doc["records"]:
        x = torch.from_numpy(rec["inputs"]["x"].view(np.int16)).view(TD[dtype]).to(cuda_device)
        bits = torch.from_numpy(np.ascontiguousarray(rec["inputs"]["bits"]).view(np.int32)).to(cuda_device)
        for variant in (0, 2):
            y = ops.bitdelta_gemm(x, bits, 0.02, variant=variant)
            torch.cuda.synchronize()
            ref = rec["refs"]["y"]
            v = compare.check(_np(y), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
            assert v.ok, (rec["case"], variant, v.summary())
    _status_ok()


TASK_SHAPES = [(128, 256, 256), (512, 4096, 4096), (100, 300, 96), (1, 64, 32)]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("shape", TASK_SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in TASK_SHAPES])
def test_task_cases(cuda_device, dtype, shape):
    m, n, k = shape
    for ci, case in enumerate(cases.BITDELTA_CASES):
        inp = cases.bitdelta_inputs(case, cases.case_seed(0, ci), m, n, k, dtype)
        x, bits = inp["x"].to(cuda_device), inp["bits"].to(cuda_device)
        y = torch.full((m, n), float("nan"), dtype=TD[dtype], device=cuda_device)
        ops.bitdelta_gemm(x, bits, 0.02, out=y)
        torch.cuda.synchronize()
        _status_ok()
        rows = np.arange(m) if m <= 64 else np.unique(np.r_[0:8, m // 2, m - 1, np.arange(0, m, max(1, m // 40))])
        ref = oref.bitdelta_gemm(_np(x)[rows], inp["bits"].numpy(), 0.02)
        v = compare.check(_np(y)[rows], ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
        assert v.ok, (case, shape, v.summary())


BASE_SHAPES = [(1, 4096, 4096), (16, 4096, 4096), (128, 4096, 4096), (3, 200, 96), (300, 256, 128)]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("shape", BASE_SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in BASE_SHAPES])
def test_base_cases(cuda_device, dtype, shape):
    m, n, k = shape
    for ci, case in enumerate(cases.BITDELTA_BASE_CASES):
        inp = cases.bitdelta_base_inputs(case, cases.case_seed(0, ci), m, n, k, dtype)
        d = {kk: v.to(cuda_device) for kk, v in inp.items()}
        y = torch.full((m, n), float("nan"), dtype=TD[dtype], device=cuda_device)
        ops.bitdelta_gemm_base(d["x"], d["w_base"], d["s_words"], d["alpha"], out=y)
        torch.cuda.synchronize()
        _status_ok()
        ref = oref.bitdelta_gemm_base(_np(d["x"]), _np(d["w_base"]), inp["s_words"].numpy(), _np(d["alpha"]))
        v = compare.check(_np(y), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
        assert v.ok, (case, shape, v.summary())


def test_base_fallback_matches(cuda_device):
    inp = cases.bitdelta_base_inputs("normal", 7919, 5, 96, 64, "fp16")
    d = {kk: v.to(cuda_device) for kk, v in inp.items()}
    y = ops.bitdelta_gemm_base(d["x"], d["w_base"], d["s_words"], d["alpha"], variant=2)
    torch.cuda.synchronize()
    ref = oref.bitdelta_gemm_base(_np(d["x"]), _np(d["w_base"]), inp["s_words"].numpy(), _np(d["alpha"]))
    assert compare.check(_np(y), ref, compare.rms_scale(ref), dtype="fp16", **TOL["fp16"]).ok


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("shape,variant", [((1, 4096, 4096), 3), ((1, 4096, 4096), 1), ((2, 300, 256), 3), ((3, 200, 96), 3),
                                           ((4, 1024, 4096), 3), ((1, 77, 32), 3)])
def test_base_streaming_and_tensor_core_variants(cuda_device, dtype, shape, variant):
    """The few-row streaming kernel (variant 3: M <= 4, a matrix-vector stream over W_base and the
    sign words) and, at M = 1, the tensor-core kernel it replaces by default (variant 1), on every
    case including planted specials, against the oracle."""
    m, n, k = shape
    for ci, case in enumerate(cases.BITDELTA_BASE_CASES):
        inp = cases.bitdelta_base_inputs(case, cases.case_seed(1, ci), m, n, k, dtype)
        d = {kk: v.to(cuda_device) for kk, v in inp.items()}
        y = torch.full((m, n), float("nan"), dtype=TD[dtype], device=cuda_device)
        ops.bitdelta_gemm_base(d["x"], d["w_base"], d["s_words"], d["alpha"], out=y, variant=variant)
        torch.cuda.synchronize()
        _status_ok()
        ref = oref.bitdelta_gemm_base(_np(d["x"]), _np(d["w_base"]), inp["s_words"].numpy(), _np(d["alpha"]))
        v = compare.check(_np(y), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
        assert v.ok, (case, shape, variant, v.summary())
