"""sf_gemm_nn_noalloc: the allocation-free form of the gemm_nn entry point.

Some callers cannot allocate device memory when they need the product — code running inside a
host callback (where CUDA API calls are forbidden), hosts whose device memory is fully reserved
by another allocator, and certified or real-time hosts that forbid allocation after start-up.
For them ``sf_gemm_nn_noalloc`` keeps the transpose scratch in a fixed device array inside the
library instead of taking a caller workspace.

This test calls the new entry point through the C ABI and checks its output against the
existing ``sf_gemm_nn`` (which takes a caller workspace) within the task tolerance used by the
other gemm tests, on two calls in a row (different shapes and data, so the second call runs on
whatever the first one left in the shared scratch).  It also checks that problems too large for
the fixed scratch are rejected.  The file is named so that pytest collects it last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from shapeforge_b200 import _native, cases, compare

pytestmark = pytest.mark.gpu

# fp16 tolerance of tasks/gemm (rtol 2e-3, atol_rel 1e-3 of the RMS scale), as in test_gemm_gpu.
RTOL, ATOL_REL = 2e-3, 1e-3
MAX_SCRATCH = 32 * 1024 * 1024


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _with_workspace(a, b, c, m, n, k):
    need = int(_native.load().sf_gemm_nn_workspace_bytes(m, n, k, 0))
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device=a.device)
    _native.call("sf_gemm_nn", a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, 0, ws.data_ptr(), ws.numel(), _stream())
    return ws


def _no_alloc(a, b, c, m, n, k):
    _native.call("sf_gemm_nn_noalloc", a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, 0, _stream())


def _inputs(m, n, k, seed, dev):
    inp = cases.gemm_inputs("normal", seed, (m, k), (k, n), "fp16")
    return inp["A"].to(dev), inp["B"].to(dev)


def test_no_alloc_matches_workspace_entry_point_twice(cuda_device):
    # Two calls in a row: the first leaves a large transposed B in the shared scratch, the
    # second (smaller, different data) must not be affected by those leftovers.
    for (m, n, k), seed in [((512, 384, 256), 101), ((256, 200, 136), 202)]:
        a, b = _inputs(m, n, k, seed, cuda_device)
        c_ref = torch.full((m, n), float("nan"), dtype=torch.float16, device=cuda_device)
        c_new = torch.full((m, n), float("nan"), dtype=torch.float16, device=cuda_device)
        ws = _with_workspace(a, b, c_ref, m, n, k)
        _no_alloc(a, b, c_new, m, n, k)
        torch.cuda.synchronize()
        del ws
        ref = c_ref.double().cpu().numpy()
        out = c_new.double().cpu().numpy()
        v = compare.check(out, ref, compare.rms_scale(ref), rtol=RTOL, atol_rel=ATOL_REL, dtype="fp16")
        assert v.ok, ((m, n, k), v.summary())
        assert not np.isnan(out).any()


def test_no_alloc_rejects_problems_larger_than_its_scratch(cuda_device):
    # K*N*2 bytes just above the fixed scratch: rejected before anything is launched.  The
    # tensors are real and large enough, so even a missed check could not read out of bounds.
    k, n, m = 4097, 4097, 1
    assert k * n * 2 > MAX_SCRATCH
    a = torch.zeros((m, k), dtype=torch.float16, device=cuda_device)
    b = torch.zeros((k, n), dtype=torch.float16, device=cuda_device)
    c = torch.zeros((m, n), dtype=torch.float16, device=cuda_device)
    with pytest.raises(_native.SfError) as exc:
        _no_alloc(a, b, c, m, n, k)
    assert exc.value.code == _native.SF_EINVAL
    assert "scratch" in exc.value.message
