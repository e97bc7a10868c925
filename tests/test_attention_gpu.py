"""flash_attention on the B200: the non-causal task contract and the causal workload.

Tolerances: the task's OpSpec ones (tasks/flash_attention/opspec.json numerics): fp16 rtol 2e-3 /
atol_rel 1e-3, bf16 rtol 1.6e-2 / atol_rel 8e-3, scaled by the RMS of the finite reference.
Large shapes compare a sample of query rows of a sample of heads (rows are independent).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

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


def _check(o, q, k, v, scale, causal, dtype, heads=None, rows=None):
    b, h, s, d = q.shape
    heads = list(range(h)) if heads is None else heads
    rows = np.arange(s) if rows is None else np.asarray(rows)
    qn, kn, vn = _np(q[:, heads]), _np(k[:, heads]), _np(v[:, heads])
    ref = oref.attention_rows(qn, kn, vn, scale, causal, rows)
    got = _np(o[:, heads])[:, :, rows]
    return compare.check(got, ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_reference_vectors(cuda_device, dtype):
    """The kernel on the reference module's q rows (placed at their positions) and full k/v."""
    doc = golden.load(f"ref_flash_attention_{dtype}")
    for rec in doc["records"]:
        full = rec["full_shapes"]["q"]
        rows = np.array(rec["slice"]["q_rows"])
        rows = np.where(rows < 0, full[2] + rows, rows)
        q = torch.zeros(full, dtype=TD[dtype])
        qs = torch.from_numpy(np.ascontiguousarray(rec["inputs"]["q"]).view(np.int16)).view(TD[dtype])
        q[:, :, torch.from_numpy(rows)] = qs
        k = torch.from_numpy(np.ascontiguousarray(rec["inputs"]["k"]).view(np.int16)).view(TD[dtype])
        v = torch.from_numpy(np.ascontiguousarray(rec["inputs"]["v"]).view(np.int16)).view(TD[dtype])
        q, k, v = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device)
        for variant in (0, 2):
            o = ops.flash_attention(q, k, v, 0.125, causal=False, variant=variant)
            torch.cuda.synchronize()
            got = _np(o)[:, :, rows]
            ref = rec["refs"]["o"]
            v_ = compare.check(got, ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
            assert v_.ok, (rec["case"], variant, v_.summary())
    _status_ok()


TASK_SHAPES = [(1, 2, 128, 64), (2, 8, 1024, 64), (1, 2, 200, 64), (1, 1, 77, 128)]


# Variants: 0 = default dispatch (a grid of at most one CTA per SM takes the kernel with S
# double-buffered in TMEM, larger grids two CTAs per SM), 1 = the two-CTA kernel, 3 = the
# double-buffered kernel at any grid.
@pytest.mark.parametrize("variant", [0, 1, 3])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("shape", TASK_SHAPES, ids=["x".join(map(str, s)) for s in TASK_SHAPES])
def test_task_cases_noncausal(cuda_device, dtype, shape, variant):
    for ci, case in enumerate(cases.ATTENTION_CASES):
        inp = cases.attention_inputs(case, cases.case_seed(0, ci), shape, dtype)
        q, k, v = (inp[n].to(cuda_device) for n in ("q", "k", "v"))
        o = torch.full_like(q, float("nan"))
        ops.flash_attention(q, k, v, 0.125, causal=False, out=o, variant=variant)
        torch.cuda.synchronize()
        _status_ok()
        heads = [0, shape[1] - 1] if shape[1] > 2 else None
        v_ = _check(o, q, k, v, 0.125, False, dtype, heads=heads)
        assert v_.ok, (case, shape, v_.summary())


CAUSAL_SHAPES = [(4, 32, 2048, 128), (4, 32, 512, 128), (4, 32, 2048, 64), (1, 2, 8192, 128), (1, 2, 300, 128), (2, 3, 129, 64)]


@pytest.mark.parametrize("variant", [0, 1, 3])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", CAUSAL_SHAPES, ids=["x".join(map(str, s)) for s in CAUSAL_SHAPES])
def test_causal_workload(cuda_device, dtype, shape, variant):
    b, h, s, d = shape
    scale = 1.0 / math.sqrt(d)
    inp = cases.attention_bench_inputs(shape, dtype, seed=cases.SEARCH_SEED)
    q, k, v = (inp[n].to(cuda_device) for n in ("q", "k", "v"))
    o = torch.full_like(q, float("nan"))
    ops.flash_attention(q, k, v, scale, causal=True, out=o, variant=variant)
    torch.cuda.synchronize()
    _status_ok()
    rng = np.random.default_rng(0)
    rows = np.unique(np.r_[0, 1, 127, 128, min(129, s - 1), s - 1, rng.choice(s, min(s, 40), replace=False)])
    heads = [0, h - 1] if h > 1 else [0]
    v_ = _check(o[:1], q[:1], k[:1], v[:1], scale, True, dtype, heads=heads, rows=rows)
    assert v_.ok, (shape, v_.summary())
    if b > 1:
        v_ = _check(o[b - 1:], q[b - 1:], k[b - 1:], v[b - 1:], scale, True, dtype, heads=[h // 2], rows=rows)
        assert v_.ok, (shape, "last batch", v_.summary())
    assert not torch.isnan(o).any()


def test_causal_fallback_matches(cuda_device):
    shape = (1, 2, 130, 64)
    inp = cases.attention_bench_inputs(shape, "bf16")
    q, k, v = (inp[n].to(cuda_device) for n in ("q", "k", "v"))
    o = ops.flash_attention(q, k, v, 0.125, causal=True, variant=2)
    torch.cuda.synchronize()
    assert _check(o, q, k, v, 0.125, True, "bf16").ok
