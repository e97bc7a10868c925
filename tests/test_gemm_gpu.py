"""GEMM on the B200 (tcgen05 kernel + general fallback) against the oracle and the reference.

Tolerances are the task's OpSpec ones (tasks/gemm/opspec.json numerics): fp16 rtol 2e-3 /
atol_rel 1e-3, bf16 rtol 1.6e-2 / atol_rel 8e-3, scaled by the RMS of the finite reference.
Large shapes compare a sample of full output rows (every row depends on all of B, so a row
sample still exercises every B tile, K block and N tile).
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


def _np(t):
    return t.detach().cpu().to(torch.float64).numpy()


def _rows_sample(m, n=48, seed=0):
    if m <= n:
        return np.arange(m)
    rng = np.random.default_rng(seed)
    pick = set(rng.choice(m, n - 4, replace=False).tolist()) | {0, 127, 128, m - 1}
    return np.array(sorted(p for p in pick if p < m))


def _check_nt(c, a, b, dtype, rows=None):
    a_np, b_np, c_np = _np(a), _np(b), _np(c)
    if rows is not None:
        a_np, c_np = a_np[rows], c_np[rows]
    ref = oref.gemm_nt(a_np, b_np)
    return compare.check(c_np, ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])


def _status_ok():
    code, where = ops.kernel_status()
    assert code == 0, f"tcgen05 kernel status {code} at wait {where}"


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_golden_vectors_nn(cuda_device, dtype):
    """The kernel on the G0 input bytes (A rows / B columns sliced) vs the reference's fp64 bytes."""
    doc = golden.load(f"g0_gemm_{dtype}")
    for rec in doc["records"]:
        a = torch.from_numpy(rec["inputs"]["A"].view(np.int16)).view(TD[dtype]).to(cuda_device)
        b = torch.from_numpy(np.ascontiguousarray(rec["inputs"]["B"]).view(np.int16)).view(TD[dtype]).to(cuda_device)
        b = b.contiguous()
        for variant in (0, 2):  # the tensor-core path (B read in place as an MN-major operand), and the fallback
            c = ops.gemm_nn(a, b, variant=variant)
            torch.cuda.synchronize()
            ref = rec["refs"]["C"]
            v = compare.check(_np(c), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
            assert v.ok, (rec["case"], variant, v.summary())
    _status_ok()


NT_SHAPES = [
    (128, 256, 64),
    (256, 512, 128),
    (512, 512, 512),       # small shard of the dense-gemm workload
    (300, 200, 72),        # ragged M/N, K tail inside a block
    (1, 256, 64),          # single row
    (129, 257, 136),       # N % 8 != 0: scalar epilogue stores
    (256, 320, 1000),      # small-problem kernel: 16 K-blocks through its 8-stage ring, K tail
    (1024, 1152, 256),     # small-problem kernel at 144 CTAs (one 128 x 64 tile per SM)
    (1024, 1216, 128),     # 152 tiles of 128 x 64: the persistent kernel again
    (4096, 4096, 4096),    # the workload
    (4095, 4096, 4096),    # tail shard
]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("shape", NT_SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in NT_SHAPES])
def test_gemm_nt_tensor_core(cuda_device, dtype, shape):
    m, n, k = shape
    case_list = cases.GEMM_CASES if m * n * k <= 512**3 else ("normal", "large", "ieee")
    for ci, case in enumerate(case_list):
        inp = cases.gemm_inputs(case, cases.case_seed(0, ci), (m, k), (n, k), dtype)
        a, b = inp["A"].to(cuda_device), inp["B"].to(cuda_device)
        c = torch.full((m, n), float("nan"), dtype=TD[dtype], device=cuda_device)
        ops.gemm_nt(a, b, out=c, variant=1)
        torch.cuda.synchronize()
        _status_ok()
        v = _check_nt(c, a, b, dtype, rows=_rows_sample(m))
        assert v.ok, (case, shape, v.summary())


FALLBACK_SHAPES = [(64, 64, 60), (33, 17, 5), (7, 130, 1)]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("shape", FALLBACK_SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in FALLBACK_SHAPES])
def test_gemm_nt_fallback_shapes(cuda_device, dtype, shape):
    """K % 8 != 0 cannot use TMA: exact dispatch routes to the general kernel."""
    m, n, k = shape
    for ci, case in enumerate(cases.GEMM_CASES):
        inp = cases.gemm_inputs(case, cases.case_seed(0, ci), (m, k), (n, k), dtype)
        a, b = inp["A"].to(cuda_device), inp["B"].to(cuda_device)
        c = ops.gemm_nt(a, b)
        torch.cuda.synchronize()
        v = _check_nt(c, a, b, dtype)
        assert v.ok, (case, shape, v.summary())
    with pytest.raises(_native.SfError):
        ops.gemm_nt(a, b, variant=1)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_gemm_nn_task_sizes(cuda_device, dtype):
    """The task contract's own tiers: small 256x256x128 and paper 2048^3 (B stored [K, N])."""
    for (m, n, k) in [(256, 256, 128), (2048, 2048, 2048)]:
        for ci, case in enumerate(cases.GEMM_CASES):
            inp = cases.gemm_inputs(case, cases.case_seed(0, ci), (m, k), (k, n), dtype)
            a, b = inp["A"].to(cuda_device), inp["B"].to(cuda_device)
            c = ops.gemm_nn(a, b)
            torch.cuda.synchronize()
            rows = _rows_sample(m)
            ref = oref.gemm_nn(_np(a)[rows], _np(b))
            v = compare.check(_np(c)[rows], ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
            assert v.ok, (case, (m, n, k), v.summary())
    _status_ok()


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_gemm_nn_direct_and_transposed(cuda_device, dtype):
    """Both tensor-core routes of the NN layout: N % 8 == 0 reads B [K, N] in place (no workspace:
    the size query returns 0); N % 8 != 0 transposes B into the caller's workspace first."""
    for (m, n, k) in [(256, 200, 136), (300, 512, 64), (256, 196, 128), (130, 20, 72)]:
        need = ops.gemm_nn_workspace_bytes(m, n, k, dtype)
        assert need == (0 if n % 8 == 0 else n * k * 2)
        inp = cases.gemm_inputs("normal", cases.case_seed(3, n), (m, k), (k, n), dtype)
        a, b = inp["A"].to(cuda_device), inp["B"].to(cuda_device)
        c = ops.gemm_nn(a, b, variant=1)
        torch.cuda.synchronize()
        ref = oref.gemm_nn(_np(a), _np(b))
        v = compare.check(_np(c), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
        assert v.ok, ((m, n, k), v.summary())
    _status_ok()


def test_k_zero_and_empty(cuda_device):
    a = torch.empty((8, 0), dtype=torch.float16, device=cuda_device)
    b = torch.empty((16, 0), dtype=torch.float16, device=cuda_device)
    c = ops.gemm_nt(a, b)
    torch.cuda.synchronize()
    assert torch.all(c == 0)
    e = ops.gemm_nt(torch.empty((0, 8), dtype=torch.float16, device=cuda_device),
                    torch.empty((4, 8), dtype=torch.float16, device=cuda_device))
    assert e.shape == (0, 4)


def test_batch_runner_gemm(cuda_device):
    m = n = k = 1024
    sets, keep = [], []
    for s in range(2):
        inp = cases.gemm_bench_inputs(m, n, k, "fp16", seed=s)
        a, b = inp["A"].to(cuda_device), inp["B"].to(cuda_device)
        c = torch.empty((m, n), dtype=torch.float16, device=cuda_device)
        keep.append((a, b, c))
        sets.append([a.data_ptr(), b.data_ptr(), c.data_ptr()])
    desc = _native.op_desc("gemm_nt", "fp16", dims=(m, n, k))
    t = _native.run_batch(desc, sets, 8, torch.cuda.current_stream().cuda_stream)
    assert t > 0
    _status_ok()
    for a, b, c in keep:
        assert _check_nt(c, a, b, "fp16", rows=_rows_sample(m)).ok
