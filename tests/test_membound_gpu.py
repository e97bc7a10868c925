"""silu, swiglu, softmax, reduction_sum and rope on the B200 against the oracle and the reference.

Tolerances are the tasks' OpSpec ones: fp16 rtol 2e-3 / atol_rel 1e-3, bf16 rtol 1.6e-2 /
atol_rel 8e-3 (reduction_sum: atol_rel 3e-6 of its error scale sum |x| per row).
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
RSUM_TOL = {"fp16": dict(rtol=2e-3, atol_rel=3e-6), "bf16": dict(rtol=1.6e-2, atol_rel=3e-6)}
TD = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _np(t):
    return t.detach().cpu().to(torch.float64).numpy()


def _dev(bits, dtype, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(TD[dtype]).to(dev)


def _run(task, inp, dtype):
    if task == "silu":
        return ops.silu(inp["x"])
    if task == "swiglu":
        return ops.swiglu(inp["gate"], inp["up"])
    if task == "softmax":
        return ops.softmax(inp["x"])
    if task == "reduction_sum":
        return ops.reduction_sum(inp["x"])
    if task == "rope":
        return ops.rope(inp["x"], 10000.0)
    raise KeyError(task)


def _oracle(task, inp):
    f = {k: _np(v) for k, v in inp.items()}
    if task == "silu":
        return oref.silu(f["x"])
    if task == "swiglu":
        return oref.swiglu(f["gate"], f["up"])
    if task == "softmax":
        return oref.softmax(f["x"])
    if task == "reduction_sum":
        return oref.reduction_sum(f["x"])
    if task == "rope":
        return oref.rope(f["x"], 10000.0)
    raise KeyError(task)


def _verdict(task, out, ref, inp, dtype):
    if task == "reduction_sum":
        scale = oref.reduction_sum_error_scale(_np(inp["x"]))
        return compare.check(_np(out), ref, scale, dtype=dtype, **RSUM_TOL[dtype])
    return compare.check(_np(out), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("task", ["softmax", "reduction_sum", "silu", "swiglu"])
def test_g0_golden_vectors(cuda_device, task, dtype):
    """The kernel on the G0 input bytes vs the reference's fp64 output bytes."""
    doc = golden.load(f"g0_{task}_{dtype}")
    for rec in doc["records"]:
        inp = {k: _dev(v, dtype, cuda_device) for k, v in rec["inputs"].items()}
        out = _run(task, inp, dtype)
        torch.cuda.synchronize()
        ref = rec["refs"]["y"]
        scale = rec["scales"]["y"]
        tol = RSUM_TOL[dtype] if task == "reduction_sum" else TOL[dtype]
        v = compare.check(_np(out), ref, scale, dtype=dtype, **tol)
        assert v.ok, (task, rec["case"], v.summary())


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_rope_reference_vectors(cuda_device, dtype):
    doc = golden.load(f"ref_rope_{dtype}")
    for rec in doc["records"]:
        x = _dev(rec["inputs"]["x"], dtype, cuda_device)
        y = ops.rope(x, 10000.0)
        torch.cuda.synchronize()
        pos = np.array(rec["slice"]["ref_positions"])
        ref = rec["refs"]["y"]
        got = _np(y)[:, :, pos]
        v = compare.check(got, ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
        assert v.ok, (rec["case"], v.summary())


SHAPES = {
    "softmax": [(8192, 2048), (64, 512), (5, 3), (3, 1000), (2, 8200), (33, 64), (9, 2040)],
    "reduction_sum": [(4096, 4096), (64, 1024), (256, 4096), (7, 13), (3, 70000)],
    "silu": [(16777216,), (65536,), (1,), (1001,)],
    "swiglu": [(16777216,), (65536,), (13,)],
    "rope": [(2, 32, 1024, 128), (1, 2, 64, 64), (1, 3, 5, 6), (2, 2, 33, 16), (1, 1, 4096, 256)],
}


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("task", sorted(SHAPES))
def test_cases_against_oracle(cuda_device, task, dtype):
    for shape in SHAPES[task]:
        for ci, case in enumerate(cases.MEMBOUND_CASES[task]):
            inp = cases.membound_inputs(task, case, cases.case_seed(0, ci), shape, dtype)
            inp = {k: v.to(cuda_device) for k, v in inp.items()}
            out = _run(task, inp, dtype)
            torch.cuda.synchronize()
            v = _verdict(task, out, _oracle(task, inp), inp, dtype)
            assert v.ok, (task, shape, case, v.summary())


@pytest.mark.parametrize("task", ["softmax", "reduction_sum", "silu", "rope"])
def test_general_kernels_match(cuda_device, task):
    """The forced general (scalar) kernel agrees with the oracle too (the portfolio fallback)."""
    shape = {"softmax": (64, 512), "reduction_sum": (64, 1024), "silu": (65536,), "rope": (1, 2, 64, 64)}[task]
    inp = cases.membound_inputs(task, "normal", 7919, shape, "fp16")
    inp = {k: v.to(cuda_device) for k, v in inp.items()}
    x = inp["x"]
    if task == "silu":
        out = ops.silu(x, variant=2)
    elif task == "softmax":
        out = ops.softmax(x, variant=2)
    elif task == "reduction_sum":
        out = ops.reduction_sum(x, variant=2)
    else:
        out = ops.rope(x, variant=2)
    torch.cuda.synchronize()
    assert _verdict(task, out, _oracle(task, inp), inp, "fp16").ok
