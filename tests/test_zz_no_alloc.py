"""sf_gemm_nn_noalloc: the allocation-free form of the gemm_nn entry point.

Some callers cannot allocate device memory when they need the product: hosts whose device
memory is fully reserved by an allocator the plug-in cannot reach, and certified or real-time
hosts that forbid allocation after start-up.  ``sf_gemm_nn`` needs a caller workspace for shapes
whose B must be transposed (N % 8 != 0); ``sf_gemm_nn_noalloc`` uses a fixed device array inside
the library instead, and runs every other shape exactly as ``sf_gemm_nn`` does.

Each call here goes through the C ABI and is checked against the oracle (fp64 ``A @ B``) within
the gemm task's tolerances, and against ``sf_gemm_nn`` with a caller workspace.  The calls run
back to back, so later calls read the shared array after earlier calls left other data there,
with a different row stride.  Every dispatch route is exercised: B read in place, B transposed
into the array, the general kernel (K % 8 != 0), K == 0, a large in-place problem beyond the
array's size (accepted: it needs no scratch) and a transposed problem beyond it (rejected).
The file is named so that pytest collects it last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import ops as oref
from shapeforge_b200 import _native, cases, compare

pytestmark = pytest.mark.gpu

# tasks/gemm/opspec.json tolerances, scaled by the RMS of the finite reference (as test_gemm_gpu).
TOL = {"fp16": dict(rtol=2e-3, atol_rel=1e-3), "bf16": dict(rtol=1.6e-2, atol_rel=8e-3)}
DT_CODE = {"fp16": 0, "bf16": 1}
TD = {"fp16": torch.float16, "bf16": torch.bfloat16}
MAX_SCRATCH = 32 * 1024 * 1024


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _np(t):
    return t.detach().cpu().to(torch.float64).numpy()


def _inputs(m, n, k, seed, dtype, dev):
    inp = cases.gemm_inputs("normal", seed, (m, k), (k, n), dtype)
    return inp["A"].to(dev), inp["B"].to(dev)


def _nan_out(m, n, dtype, dev):
    return torch.full((m, n), float("nan"), dtype=TD[dtype], device=dev)


def _no_alloc(a, b, c, m, n, k, dtype):
    _native.call("sf_gemm_nn_noalloc", a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, DT_CODE[dtype], _stream())


def _with_workspace(a, b, c, m, n, k, dtype):
    need = int(_native.load().sf_gemm_nn_workspace_bytes(m, n, k, DT_CODE[dtype]))
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=a.device)
    _native.call("sf_gemm_nn", a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, DT_CODE[dtype], ws.data_ptr(), ws.numel(),
                 _stream())
    return ws


def _check(out, ref, dtype, what):
    v = compare.check(out, ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])
    assert v.ok, (what, v.summary())
    assert not np.isnan(out).any(), what


# (M, N, K), dtype, seed, route.  Consecutive transposed calls leave [N, K] images of different
# row strides in the shared array, so each one reads over the previous call's leftovers.
SEQUENCE = [
    ((512, 384, 256), "fp16", 101, "in place"),
    ((256, 203, 1024), "fp16", 202, "transposed"),
    ((128, 301, 520), "bf16", 303, "transposed"),
    ((64, 203, 130), "fp16", 404, "general kernel"),
    ((192, 77, 96), "bf16", 505, "transposed"),
    ((256, 200, 136), "bf16", 606, "in place"),
]


def test_no_alloc_matches_oracle_and_workspace_entry_point(cuda_device):
    for (m, n, k), dtype, seed, route in SEQUENCE:
        a, b = _inputs(m, n, k, seed, dtype, cuda_device)
        c_new = _nan_out(m, n, dtype, cuda_device)
        c_ws = _nan_out(m, n, dtype, cuda_device)
        _no_alloc(a, b, c_new, m, n, k, dtype)
        ws = _with_workspace(a, b, c_ws, m, n, k, dtype)
        torch.cuda.synchronize()
        del ws
        what = ((m, n, k), dtype, route)
        out = _np(c_new)
        _check(out, oref.gemm_nn(_np(a), _np(b)), dtype, what)
        _check(out, _np(c_ws), dtype, what)


def test_no_alloc_called_twice_in_a_row_gives_the_same_answer(cuda_device):
    # Two transposed calls in a row on the same inputs, with another shape in between that
    # overwrites the shared array: the answers agree bit for bit.
    m, n, k = 320, 203, 512
    a, b = _inputs(m, n, k, 707, "fp16", cuda_device)
    first, second = _nan_out(m, n, "fp16", cuda_device), _nan_out(m, n, "fp16", cuda_device)
    _no_alloc(a, b, first, m, n, k, "fp16")
    a2, b2 = _inputs(96, 333, 264, 808, "fp16", cuda_device)
    _no_alloc(a2, b2, _nan_out(96, 333, "fp16", cuda_device), 96, 333, 264, "fp16")
    _no_alloc(a, b, second, m, n, k, "fp16")
    torch.cuda.synchronize()
    assert torch.equal(first, second)
    _check(_np(first), oref.gemm_nn(_np(a), _np(b)), "fp16", "repeat")


def test_no_alloc_k0_writes_zeros(cuda_device):
    m, n = 64, 203
    a = torch.empty((m, 0), dtype=torch.float16, device=cuda_device)
    b = torch.empty((0, n), dtype=torch.float16, device=cuda_device)
    c = _nan_out(m, n, "fp16", cuda_device)
    # Zero-size tensors may have null data pointers; pass real (unused) ones for A and B.
    dummy = torch.zeros(16, dtype=torch.float16, device=cuda_device)
    _native.call("sf_gemm_nn_noalloc", dummy.data_ptr(), dummy.data_ptr(), c.data_ptr(), m, n, 0, 0, _stream())
    torch.cuda.synchronize()
    assert torch.equal(c, torch.zeros_like(c))
    del a, b


def test_no_alloc_in_place_shape_beyond_scratch_is_accepted(cuda_device):
    # N % 8 == 0: B is read in place, so K*N*2 = 64 MiB (twice the array) needs no scratch.
    m, n, k = 128, 8192, 4096
    assert k * n * 2 > MAX_SCRATCH
    a, b = _inputs(m, n, k, 909, "fp16", cuda_device)
    c = _nan_out(m, n, "fp16", cuda_device)
    _no_alloc(a, b, c, m, n, k, "fp16")
    torch.cuda.synchronize()
    rows = np.array([0, 1, 63, 64, 127])
    ref = oref.gemm_nn(_np(a)[rows], _np(b))
    _check(_np(c)[rows], ref, "fp16", "in place beyond scratch")


def test_no_alloc_rejects_transposed_problems_larger_than_its_scratch(cuda_device):
    # N % 8 != 0 with K*N*2 bytes just above the array: rejected before anything is launched.
    # The tensors are real and large enough, so even a missed check could not read out of bounds.
    k, n, m = 4096, 4100, 1
    assert n % 8 != 0 and k * n * 2 > MAX_SCRATCH
    a = torch.zeros((m, k), dtype=torch.float16, device=cuda_device)
    b = torch.zeros((k, n), dtype=torch.float16, device=cuda_device)
    c = torch.zeros((m, n), dtype=torch.float16, device=cuda_device)
    with pytest.raises(_native.SfError) as exc:
        _no_alloc(a, b, c, m, n, k, "fp16")
    assert exc.value.code == _native.SF_EINVAL
    assert "scratch" in exc.value.message
