"""mamba2_chunk_scan on the B200 against the reference's vectors and the fp64 oracle.

Tolerances: the task's OpSpec ones (tasks/mamba2_chunk_scan/opspec.json numerics): fp16
rtol 2e-3 / atol_rel 1e-3, bf16 rtol 1.6e-2 / atol_rel 8e-3, scaled by the RMS of the finite
reference; NaN/Inf must land exactly where the reference has them.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops as oref
from shapeforge_b200 import _native, cases, compare, ops
from tests import golden

pytestmark = pytest.mark.gpu

TOL = {"fp16": dict(rtol=2e-3, atol_rel=1e-3), "bf16": dict(rtol=1.6e-2, atol_rel=8e-3)}
TD = {"fp16": torch.float16, "bf16": torch.bfloat16}
NAMES = ("x", "dt", "dA_cumsum", "Bmat", "Cmat", "Dskip", "states")


def _np(t):
    return t.detach().cpu().to(torch.float64).numpy()


def _status_ok():
    code, where = ops.kernel_status()
    assert code == 0, f"tensor-core kernel status {code} at wait {where}"


def _run(inp, dev, variant=0):
    t = [inp[n].to(dev) for n in NAMES]
    y = torch.full_like(t[0], float("nan"))
    ops.mamba2_chunk_scan(*t, out=y, variant=variant)
    torch.cuda.synchronize()
    return y


def _oracle(inp):
    return oref.mamba2_chunk_scan(*[inp[n].to(torch.float64).numpy() for n in NAMES])


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_reference_vectors(cuda_device, dtype):
    """The reference module's inputs (first and last chunk of the small size) through both kernels."""
    doc = golden.load(f"ref_mamba2_chunk_scan_{dtype}")
    for rec in doc["records"]:
        inp = {n: torch.from_numpy(np.ascontiguousarray(rec["inputs"][n]).view(np.int16)).view(TD[dtype]) for n in NAMES}
        rows = np.array(rec["slice"]["ref_rows"])
        ref = rec["refs"]["y"]
        for variant in (0, 2):
            y = _run(inp, cuda_device, variant)
            v = compare.check(_np(y)[:, rows], ref, float(rec["scales"]["y"]), dtype=dtype, **TOL[dtype])
            assert v.ok, (rec["case"], variant, v.summary())
    _status_ok()


SHAPES = {
    "small": (1, 256, 2, 64, 64, 64),
    "paper": (2, 2048, 8, 64, 64, 64),
    "odd_chunks": (3, 192, 5, 64, 64, 64),
    "one_chunk": (2, 64, 3, 64, 64, 64),
}


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("size", list(SHAPES))
def test_task_cases(cuda_device, dtype, size):
    b, l, h, p, n, c = SHAPES[size]
    for ci, case in enumerate(cases.MAMBA2_CASES):
        inp = cases.mamba2_inputs(case, cases.case_seed(0, ci), b, l, h, p, n, c, dtype)
        ref = _oracle(inp)
        y = _run(inp, cuda_device)
        _status_ok()
        v = compare.check(_np(y), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
        assert v.ok, (size, case, v.summary())


GENERAL = [(1, 96, 3, 32, 16, 32), (2, 200, 2, 24, 40, 100), (1, 400, 1, 16, 8, 200), (1, 128, 2, 64, 64, 64)]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("shape", GENERAL, ids=["x".join(map(str, s)) for s in GENERAL])
def test_general_kernel(cuda_device, dtype, shape):
    """Shapes the tensor-core kernel does not take (and one it does, forced general)."""
    b, l, h, p, n, c = shape
    for ci, case in enumerate(("normal", "wide_range", "ieee")):
        inp = cases.mamba2_inputs(case, cases.case_seed(3, ci), b, l, h, p, n, c, dtype)
        ref = _oracle(inp)
        y = _run(inp, cuda_device, variant=2)
        v = compare.check(_np(y), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
        assert v.ok, (shape, case, v.summary())


@pytest.mark.parametrize("variant", [0, 2])
def test_nonfinite_x_stays_in_its_chunk(cuda_device, variant):
    """A masked weight is an exact zero that still multiplies x: an inf in x makes every row of
    its chunk NaN/inf in that column and nothing else, including the other chunk of a CTA pair."""
    inp = cases.mamba2_inputs("normal", 17, 1, 256, 2, 64, 64, 64, "bf16")
    inp["x"][0, 64 + 40, 1, 3] = float("inf")
    ref = _oracle(inp)
    y = _run(inp, cuda_device, variant)
    _status_ok()
    got = _np(y)
    assert np.array_equal(~np.isfinite(got), ~np.isfinite(ref))
    v = compare.check(got, ref, compare.rms_scale(ref), dtype="bf16", **TOL["bf16"])
    assert v.ok, v.summary()


def test_misaligned_takes_general_path(cuda_device):
    b, l, h, p, n, c = 1, 128, 2, 64, 64, 64
    inp = cases.mamba2_inputs("normal", 23, b, l, h, p, n, c, "fp16")
    t = {k: v.to(cuda_device) for k, v in inp.items()}
    raw = torch.empty(t["x"].numel() + 1, dtype=torch.float16, device=cuda_device)
    x_mis = raw[1:].view(t["x"].shape)
    x_mis.copy_(t["x"])
    y = ops.mamba2_chunk_scan(x_mis, *[t[k] for k in NAMES[1:]])
    torch.cuda.synchronize()
    ref = _oracle(inp)
    v = compare.check(_np(y), ref, compare.rms_scale(ref), dtype="fp16", **TOL["fp16"])
    assert v.ok, v.summary()
    with pytest.raises(_native.SfError):
        ops.mamba2_chunk_scan(x_mis, *[t[k] for k in NAMES[1:]], variant=1)


def test_empty_batch_is_a_no_op(cuda_device):
    inp = cases.mamba2_inputs("normal", 1, 1, 64, 1, 64, 64, 64, "fp16")
    t = {k: v[:0].to(cuda_device) if k in ("x", "dt", "dA_cumsum", "Bmat", "Cmat", "states") else v.to(cuda_device)
         for k, v in inp.items()}
    y = ops.mamba2_chunk_scan(*[t[k] for k in NAMES])
    torch.cuda.synchronize()
    assert y.numel() == 0
