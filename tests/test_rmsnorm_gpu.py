"""rmsnorm on the B200 through the C ABI, against the oracle and the reference's golden outputs.

Tolerances are the task's OpSpec ones (tasks/rmsnorm/opspec.json:71-81): fp16 rtol 2e-3 /
atol_rel 1e-3, bf16 rtol 1.6e-2 / atol_rel 8e-3, scaled by the RMS of the finite reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle import ops as oref
from shapeforge_b200 import _native, cases, compare, ops
from tests import golden

pytestmark = pytest.mark.gpu

TOL = {"fp16": dict(rtol=2e-3, atol_rel=1e-3), "bf16": dict(rtol=1.6e-2, atol_rel=8e-3)}
TD = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().to(torch.float64).numpy()


def _verdict(y, x, w, dtype, eps=1e-6):
    ref = oref.rmsnorm(_np(x), _np(w), eps)
    return compare.check(_np(y), ref, compare.rms_scale(ref), dtype=dtype, **TOL[dtype])


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_golden_vectors(cuda_device, dtype):
    """The kernel on the G0 input bytes, compared with the reference's own fp64 output bytes."""
    doc = golden.load(f"g0_rmsnorm_{dtype}")
    for rec in doc["records"]:
        x = torch.from_numpy(rec["inputs"]["x"].view(np.int16)).view(TD[dtype]).to(cuda_device)
        w = torch.from_numpy(rec["inputs"]["w"].view(np.int16)).view(TD[dtype]).to(cuda_device)
        y = ops.rmsnorm(x, w, 1e-6)
        torch.cuda.synchronize()
        ref = rec["refs"]["y"]
        scale = float(rec["scales"]["y"])
        v = compare.check(_np(y), ref, scale, dtype=dtype, **TOL[dtype])
        assert v.ok, (rec["case"], v.summary())


SHAPES = [
    (64, 512),      # small tier (a warp per row)
    (4096, 1024),   # portfolio shards of the rmsnorm workload (a warp per row, four vectors per lane)
    (1000, 8),      # one vector per row: 31 lanes of every warp masked
    (33, 1016),     # 127 vectors: the last lane's fourth vector masked
    (4096, 4096),
    (4096, 8192),
    (4093, 4096),   # tail rows
    (3, 7),         # hidden not a multiple of 8: general kernel
    (5, 520),       # 65 vectors: masked threads
    (2, 65536),     # NV = 8 with 1024 threads
    (1, 65544),     # past the vector limit: general kernel
    (0, 128),       # empty
]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{r}x{h}" for r, h in SHAPES])
def test_cases_against_oracle(cuda_device, dtype, shape):
    rows, hidden = shape
    for ci, case in enumerate(cases.RMSNORM_CASES):
        inp = cases.rmsnorm_inputs(case, cases.case_seed(0, ci), rows, hidden, dtype)
        x, w = inp["x"].to(cuda_device), inp["w"].to(cuda_device)
        y = torch.full_like(x, float("nan"))  # poisoned output: every element must be written
        ops.rmsnorm(x, w, 1e-6, out=y)
        torch.cuda.synchronize()
        v = _verdict(y, x, w, dtype)
        assert v.ok, (case, shape, v.summary())


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_misaligned_rows_use_the_general_kernel(cuda_device, dtype):
    """A view starting 2 bytes into an allocation is not 16-byte aligned."""
    rows, hidden = 16, 256
    inp = cases.rmsnorm_inputs("normal", 11, rows, hidden + 1, dtype)
    base = inp["x"].to(cuda_device).reshape(-1)
    x = base[1 : 1 + rows * hidden].view(rows, hidden)
    w = inp["w"][:hidden].to(cuda_device)
    y = ops.rmsnorm(x, w, 1e-6)
    torch.cuda.synchronize()
    assert _verdict(y, x, w, dtype).ok


def test_run_op_and_batch_through_the_c_abi(cuda_device):
    rows, hidden = 256, 4096
    sets = []
    tensors = []
    for s in range(3):
        inp = cases.rmsnorm_bench_inputs(rows, hidden, "fp16", seed=s)
        x, w = inp["x"].to(cuda_device), inp["w"].to(cuda_device)
        y = torch.empty_like(x)
        tensors.append((x, w, y))
        sets.append([x.data_ptr(), w.data_ptr(), y.data_ptr()])
    desc = _native.op_desc("rmsnorm", "fp16", dims=(rows, hidden), attrs=(1e-6,))
    stream = torch.cuda.current_stream().cuda_stream
    _native.run_op(desc, sets[0], stream)
    t_plain = _native.run_batch(desc, sets, 12, stream)
    t_graph = _native.run_batch(desc, sets, 12, stream, use_graph=True)
    assert t_plain > 0 and t_graph > 0
    for x, w, y in tensors:
        assert _verdict(y, x, w, "fp16").ok
