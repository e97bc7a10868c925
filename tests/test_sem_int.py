"""sem_int: the CUDA renderer of the int32 program documents.

CPU: every program renders and compiles for sm_100a.  GPU: the compiled kernels are bit-exact
(the tasks declare ``exact: true``) against the reference's outputs and the oracle."""

from __future__ import annotations

import numpy as np
import pytest

from shapeforge_b200 import candidates, sem_int
from tests import golden

TASKS = ["sem_int_1", "sem_int_2", "sem_int_3", "sem_int_4", "sem_int_5", "sem_int_7"]


@pytest.mark.parametrize("task", TASKS)
def test_render_and_compile(task):
    doc = golden.load(f"ref_{task}_i32")["program"]
    src = sem_int.render_cuda(doc)
    assert 'extern "C" __global__' in src and sem_int.KERNEL_NAME in src
    image = candidates.compile_source(src, name=task)
    assert len(image) > 1000


def test_renderer_refuses_unregistered_rules():
    doc = golden.load("ref_sem_int_1_i32")["program"]
    bad = dict(doc, rules=dict(doc["rules"], wrap_kinds=["bin"]))
    with pytest.raises(ValueError):
        sem_int.render_cuda(bad)
    with pytest.raises(ValueError):
        sem_int.render_cuda(dict(doc, statements=[{"kind": "div", "dst": "t1", "a": "xv"}]))


@pytest.mark.gpu
@pytest.mark.parametrize("task", TASKS)
def test_bit_exact_on_reference_vectors(cuda_device, task):
    import torch

    from oracle import sem_int as oracle_sem_int
    from shapeforge_b200 import cases

    doc = golden.load(f"ref_{task}_i32")
    prog = sem_int.SemIntProgram(doc["program"])
    for rec in doc["records"]:
        x = torch.from_numpy(rec["inputs"]["x"].astype(np.int32)).to(cuda_device)
        y = torch.from_numpy(rec["inputs"]["y"].astype(np.int32)).to(cuda_device)
        out = torch.full_like(x, -1)
        prog.run(x, y, out, 12345)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().astype(np.int64), rec["refs"]["out"].astype(np.int64)), (task, rec["case"])
    # paper size (N = 65536) on the three case streams, against the oracle
    g = torch.Generator().manual_seed(cases.case_seed(0, 0))
    for lo, hi in ((-(1 << 31), 1 << 31), (-50, 50)):
        x = torch.randint(lo, hi, (65536,), generator=g, dtype=torch.int64).to(torch.int32)
        y = torch.randint(lo, hi, (65536,), generator=g, dtype=torch.int64).to(torch.int32)
        out = torch.empty_like(x, device=cuda_device)
        prog.run(x.to(cuda_device), y.to(cuda_device), out, 12345)
        torch.cuda.synchronize()
        ref = oracle_sem_int.evaluate(doc["program"], x.numpy(), y.numpy(), 12345)
        assert np.array_equal(out.cpu().numpy(), ref), task
