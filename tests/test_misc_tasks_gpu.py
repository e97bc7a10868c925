"""relu, sigmoid, sigmoid_shift, lion, gemv and gemm_silu on the B200 against the reference and the oracle.

Each task is checked three ways:

* on the reference's own inputs and fp64 outputs (``tests/golden/ref_<task>_<dtype>.npz``, written
  by ``tests/golden/make_fixtures.py`` from tasks/<task>/reference.py), with the recorded error
  scales (lion: the task's ``error_scale`` hook, per element);
* on the task's input streams (restated in ``shapeforge_b200.cases``) at the reference's small and
  paper sizes and at ragged sizes, against the oracle;
* through the forced general kernels (variant 2) on a few shapes.

Tolerances are the tasks' OpSpec ones: fp16 rtol 2e-3 / atol_rel 1e-3, bf16 rtol 1.6e-2 /
atol_rel 8e-3.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops as oref
from shapeforge_b200 import cases, compare, ops
from tests import golden

pytestmark = pytest.mark.gpu

TOL = {"fp16": dict(rtol=2e-3, atol_rel=1e-3), "bf16": dict(rtol=1.6e-2, atol_rel=8e-3)}
TD = {"fp16": torch.float16, "bf16": torch.bfloat16}
UNARY = ("relu", "sigmoid", "sigmoid_shift")
L = cases.LION_DEFAULTS


def _np(t):
    return t.detach().cpu().to(torch.float64).numpy()


def _dev(bits, dtype, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(TD[dtype]).to(dev)


def _unary(task, x, variant=0):
    return getattr(ops, task)(x, variant=variant)


def _lion_check(p, g, m, p_out, m_out, dtype, p_ref=None, m_ref=None, scales=None):
    """Compare a Lion step with the fp64 reference under the task's own error scale."""
    f = [_np(t) for t in (p, g, m)]
    if p_ref is None:
        p_ref, m_ref = oref.lion(*f, L["LR"], L["WD"], L["BETA1"], L["BETA2"])
    if scales is None:
        scales = oref.lion_error_scale(*f, p_ref, m_ref, L["LR"], L["BETA1"], TOL[dtype]["atol_rel"])
    vp = compare.check(_np(p_out), p_ref, scales[0], dtype=dtype, **TOL[dtype])
    vm = compare.check(_np(m_out), m_ref, scales[1], dtype=dtype, **TOL[dtype])
    return vp, vm


def _status_ok():
    code, where = ops.kernel_status()
    assert code == 0, f"tcgen05 kernel status {code} at wait {where}"


# ---- the reference's own vectors ---------------------------------------------------------------


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("task", UNARY)
def test_unary_reference_vectors(cuda_device, task, dtype):
    doc = golden.load(f"ref_{task}_{dtype}")
    assert len(doc["records"]) == 6
    for rec in doc["records"]:
        x = _dev(rec["inputs"]["x"], dtype, cuda_device)
        for variant in (0, 2):
            y = _unary(task, x, variant)
            torch.cuda.synchronize()
            v = compare.check(_np(y), rec["refs"]["y"], rec["scales"]["y"], dtype=dtype, **TOL[dtype])
            assert v.ok, (task, rec["case"], variant, v.summary())


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_lion_reference_vectors(cuda_device, dtype):
    doc = golden.load(f"ref_lion_{dtype}")
    a = doc["attrs"]
    for rec in doc["records"]:
        p, g, m = (_dev(rec["inputs"][k], dtype, cuda_device) for k in ("p", "g", "m"))
        for variant in (0, 2):
            p_out, m_out = ops.lion(p, g, m, a["LR"], a["WD"], a["BETA1"], a["BETA2"], variant=variant)
            torch.cuda.synchronize()
            scales = (rec["scales"]["p_out"], rec["scales"]["m_out"])
            vp, vm = _lion_check(p, g, m, p_out, m_out, dtype, rec["refs"]["p_out"], rec["refs"]["m_out"], scales)
            assert vp.ok, (rec["case"], variant, "p_out", vp.summary())
            assert vm.ok, (rec["case"], variant, "m_out", vm.summary())


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_gemv_reference_vectors(cuda_device, dtype):
    doc = golden.load(f"ref_gemv_{dtype}")
    for rec in doc["records"]:
        a = _dev(rec["inputs"]["A"], dtype, cuda_device)
        x = _dev(rec["inputs"]["x"], dtype, cuda_device)
        for variant in (0, 2):
            y = ops.gemv(a, x, variant=variant)
            torch.cuda.synchronize()
            v = compare.check(_np(y), rec["refs"]["y"], rec["scales"]["y"], dtype=dtype, **TOL[dtype])
            assert v.ok, (rec["case"], variant, v.summary())


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_gemm_silu_reference_vectors(cuda_device, dtype):
    """The sliced B has a column count that is not a multiple of 8: the tensor-core kernel runs on
    the transposed workspace copy (variant 0), and the general kernel (variant 2) is checked too."""
    doc = golden.load(f"ref_gemm_silu_{dtype}")
    for rec in doc["records"]:
        a = _dev(rec["inputs"]["A"], dtype, cuda_device)
        b = _dev(rec["inputs"]["B"], dtype, cuda_device)
        for variant in (0, 2):
            c = ops.gemm_silu(a, b, variant=variant)
            torch.cuda.synchronize()
            v = compare.check(_np(c), rec["refs"]["C"], rec["scales"]["C"], dtype=dtype, **TOL[dtype])
            assert v.ok, (rec["case"], variant, v.summary())
    _status_ok()


# ---- the task streams against the oracle --------------------------------------------------------

UNARY_SIZES = [16777216, 65536, 1, 13, 1001]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("task", UNARY)
def test_unary_cases_against_oracle(cuda_device, task, dtype):
    fn = {"relu": oref.relu, "sigmoid": oref.sigmoid, "sigmoid_shift": oref.sigmoid_shift}[task]
    for n in UNARY_SIZES:
        for ci, case in enumerate(cases.MEMBOUND_CASES[task]):
            x = cases.membound_inputs(task, case, cases.case_seed(0, ci), (n,), dtype)["x"].to(cuda_device)
            y = _unary(task, x)
            torch.cuda.synchronize()
            ref = fn(_np(x))
            v = compare.check(_np(y), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
            assert v.ok, (task, n, case, v.summary())


def test_relu_is_exact_and_keeps_nan(cuda_device):
    """relu rounds nothing: every output is the input or +0 bit for bit, NaN stays NaN and -0 -> +0."""
    for dtype in ("fp16", "bf16"):
        x = cases.membound_inputs("relu", "ieee", 11, (1 << 20,), dtype)["x"]
        x[:4] = torch.tensor([-0.0, 0.0, float("nan"), float("-inf")], dtype=x.dtype)
        y = ops.relu(x.to(cuda_device)).cpu()
        xb, yb = x.view(torch.int16), y.view(torch.int16)
        keep = x > 0
        assert torch.equal(yb[keep], xb[keep])
        nan = torch.isnan(x)
        assert torch.isnan(y[nan]).all()
        zero = ~keep & ~nan
        assert (yb[zero] == 0).all()


LION_SIZES = [8388608, 65536, 13, 1]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_lion_cases_against_oracle(cuda_device, dtype):
    for n in LION_SIZES:
        for ci, case in enumerate(cases.LION_CASES):
            inp = {k: v.to(cuda_device) for k, v in cases.lion_inputs(case, cases.case_seed(0, ci), n, dtype).items()}
            p_out, m_out = ops.lion(inp["p"], inp["g"], inp["m"], L["LR"], L["WD"], L["BETA1"], L["BETA2"])
            torch.cuda.synchronize()
            vp, vm = _lion_check(inp["p"], inp["g"], inp["m"], p_out, m_out, dtype)
            assert vp.ok, (n, case, "p_out", vp.summary())
            assert vm.ok, (n, case, "m_out", vm.summary())


# Aligned K % 8 == 0 shapes take the vector kernel (including a ragged row count and K = 8 / 8192);
# the rest take the scalar loop.
GEMV_SHAPES = [(4096, 4096), (1501, 8192), (1024, 8), (2048, 2056), (256, 512), (1, 8), (7, 13), (300, 1000), (33, 2056),
               (2, 65536)]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_gemv_cases_against_oracle(cuda_device, dtype):
    for m, k in GEMV_SHAPES:
        for ci, case in enumerate(cases.GEMV_CASES):
            inp = {kk: v.to(cuda_device) for kk, v in cases.gemv_inputs(case, cases.case_seed(0, ci), m, k, dtype).items()}
            y = ops.gemv(inp["A"], inp["x"])
            torch.cuda.synchronize()
            ref = oref.gemv(_np(inp["A"]), _np(inp["x"]))
            v = compare.check(_np(y), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
            assert v.ok, ((m, k), case, v.summary())


def test_gemv_kernels_agree(cuda_device):
    """The vector kernel (variants 0 and 1) and the scalar loop (variant 2) meet the tolerance on
    the same inputs (the ieee case: specials planted in A)."""
    inp = {k: v.to(cuda_device) for k, v in cases.gemv_inputs("ieee", 31, 4096, 4096, "bf16").items()}
    ref = oref.gemv(_np(inp["A"]), _np(inp["x"]))
    for variant in (0, 1, 2):
        y = ops.gemv(inp["A"], inp["x"], variant=variant)
        torch.cuda.synchronize()
        v = compare.check(_np(y), ref, compare.rms_scale(ref), dtype="bf16", **TOL["bf16"])
        assert v.ok, (variant, v.summary())
    code, where = ops.kernel_status()
    assert code == 0, (code, where)


def test_gemv_unaligned_and_k_zero(cuda_device):
    """An unaligned A view takes the scalar loop; K == 0 writes +0."""
    inp = cases.gemv_inputs("normal", 5, 64, 257, "fp16")
    buf = torch.empty(64 * 256 + 1, dtype=torch.float16, device=cuda_device)
    a = buf[1:].view(64, 256)
    a.copy_(inp["A"][:, :256].to(cuda_device))
    x = inp["x"][:256].to(cuda_device)
    y = ops.gemv(a, x)
    torch.cuda.synchronize()
    ref = oref.gemv(_np(a), _np(x))
    assert compare.check(_np(y), ref, compare.rms_scale(ref), dtype="fp16", **TOL["fp16"]).ok
    y0 = ops.gemv(torch.empty((5, 0), dtype=torch.float16, device=cuda_device),
                  torch.empty((0,), dtype=torch.float16, device=cuda_device))
    torch.cuda.synchronize()
    assert torch.equal(y0.view(torch.int16).cpu(), torch.zeros(5, dtype=torch.int16))


GEMM_SILU_SHAPES = [
    (2048, 2048, 2048),  # the paper size (row sample compared)
    (256, 256, 128),     # the small size
    (300, 512, 64),      # ragged M
    (130, 20, 72),       # N % 8 != 0: transposed workspace
    (129, 257, 136),     # N % 8 != 0, ragged everything
    (64, 64, 0),         # K == 0: silu(0) = 0
]


def _rows_sample(m, n=48, seed=0):
    if m <= n:
        return np.arange(m)
    rng = np.random.default_rng(seed)
    pick = set(rng.choice(m, n - 4, replace=False).tolist()) | {0, 127, 128, m - 1}
    return np.array(sorted(p for p in pick if p < m))


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_gemm_silu_cases_against_oracle(cuda_device, dtype):
    for m, n, k in GEMM_SILU_SHAPES:
        for ci, case in enumerate(cases.GEMM_SILU_CASES):
            if k == 0 and case != "normal":
                continue
            inp = cases.gemm_inputs(case, cases.case_seed(0, ci), (m, k), (k, n), dtype)
            a, b = inp["A"].to(cuda_device), inp["B"].to(cuda_device)
            c = ops.gemm_silu(a, b)
            torch.cuda.synchronize()
            rows = _rows_sample(m)
            ref = oref.gemm_silu(_np(a)[rows], _np(b))
            v = compare.check(_np(c)[rows], ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
            assert v.ok, ((m, n, k), case, v.summary())
    _status_ok()


def test_gemm_silu_paths_agree(cuda_device):
    """Every path (0 dispatch, 1 forced tensor core, 2 general kernel) meets the tolerance on a
    shape whose N % 8 == 0 (B read in place)."""
    inp = cases.gemm_inputs("normal", 3, (512, 256), (256, 264), "bf16")
    a, b = inp["A"].to(cuda_device), inp["B"].to(cuda_device)
    ref = oref.gemm_silu(_np(a), _np(b))
    for variant in (0, 1, 2):
        c = ops.gemm_silu(a, b, variant=variant)
        torch.cuda.synchronize()
        v = compare.check(_np(c), ref, compare.rms_scale(ref), dtype="bf16", **TOL["bf16"])
        assert v.ok, (variant, v.summary())
    _status_ok()
