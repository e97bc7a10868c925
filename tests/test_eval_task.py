"""The eval-v2 path on the host: a task directory's opspec and reference.py become the evaluator's
request (ABI specs, seeded cases, fp64 references, scales, tolerances, symbol arguments), and a
candidate that does not build ends as a typed compile_error report from the supervised worker —
all before anything reaches a GPU."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from shapeforge_b200 import eval_task

ROOT = Path(__file__).resolve().parents[1]
TASK = ROOT / "tasks" / "gemm_nt"

BROKEN = '''extern "C" __global__ void gemm_nt(const __half* A, const __half* B, __half* C, long long M, long long N,
                                   long long K) {
    C[0] = A[0]
}
/* taic-launch
kernel gemm_nt grid=1 threads=32
*/
'''


def test_prepare_builds_the_request_from_the_task_directory():
    req = eval_task.prepare(TASK, "fp16", "small", cases=["normal", "ieee"])
    m, n, k = (req["names"][s] for s in ("M", "N", "K"))
    assert [(s.name, s.shape, s.dtype, s.role) for s in req["specs"]] == [
        ("A", (m, k), torch.float16, "input"), ("B", (n, k), torch.float16, "input"), ("C", (m, n), torch.float16, "output")]
    assert [c.value for c in req["scalars"]] == [req["names"][s] for s in ("M", "N", "K")]
    assert (req["rtol"], req["atol_rel"], req["exact"]) == (0.002, 0.001, False)
    (c0, inputs, refs, scales), (c1, inputs1, _, _) = req["cases"]
    assert (c0, c1) == ("normal", "ieee")
    a, b = (inputs[x].double().numpy() for x in "AB")
    np.testing.assert_allclose(refs["C"], a @ b.T, rtol=1e-12, atol=1e-12)  # fp64 on the rounded inputs
    assert scales["C"] > 0 and not torch.isfinite(inputs1["A"]).all()  # the ieee case plants specials
    # Case i is seeded seed + 7919 (i + 1): a single-case request reproduces case 0.
    again = eval_task.prepare(TASK, "fp16", "small", cases=["normal"])["cases"][0][1]["A"]
    assert torch.equal(again, inputs["A"])


def test_a_candidate_that_does_not_build_is_a_compile_error(tmp_path, capsys):
    kernel = tmp_path / "k.cu"
    kernel.write_text(BROKEN)
    rc = eval_task.main([str(TASK), str(kernel), "--cases", "normal", "--in-process"])
    rep = json.loads(capsys.readouterr().out)
    assert rc == 1 and rep["status"] == "compile_error" and "expected a" in rep["detail"]
    rc = eval_task.main([str(TASK), str(kernel), "--cases", "normal", "--timeout", "300"])  # supervised worker
    rep = json.loads(capsys.readouterr().out)
    assert rc == 1 and rep["status"] == "compile_error", rep


def test_prepare_reads_the_reference_task_directories():
    """The reference's own task directories (skipped when its checkout is not mounted): attribute
    defaults, the lion error_scale hook's per-element scales, integer exactness, varlen offsets."""
    import os

    import pytest

    tasks = Path(os.environ.get("REFERENCE_ROOT", "/root/reference")) / "tasks"
    if not (tasks / "rmsnorm" / "opspec.json").is_file():
        pytest.skip("reference checkout not mounted")
    rms = eval_task.prepare(tasks / "rmsnorm", "bf16", "small", cases=["normal"])
    (_, inputs, refs, _), = rms["cases"]
    x, w = (inputs[k].double().numpy() for k in "xw")
    np.testing.assert_allclose(refs["y"], x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * w, rtol=1e-12)
    assert (rms["rtol"], rms["atol_rel"]) == (0.016, 0.008)
    lion = eval_task.prepare(tasks / "lion", "fp16", "small", cases=["normal"])
    scales = lion["cases"][0][3]
    assert scales["p_out"].shape == lion["specs"][0].shape and np.ndim(scales["m_out"]) == 0
    sem = eval_task.prepare(tasks / "sem_int_1", "i32", "small", cases=None)
    assert sem["exact"] and all(s.dtype == torch.int32 for s in sem["specs"])
    varlen = eval_task.prepare(tasks / "varlen_kda", "fp16", "mixed", cases=["canonical"])
    cu = varlen["cases"][0][1]["cu_seqlens"].tolist()
    assert cu[0] == 0 and cu[-1] == varlen["specs"][0].shape[0] and cu == sorted(cu)
