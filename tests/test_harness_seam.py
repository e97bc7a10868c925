"""The reference's own v2 evaluation seam driven by this backend (host side).

``tcenv.taskcontract.runner.evaluate_task`` (runner.py:553) is called with this repository's
``HarnessBuilder`` (a real nvcc build returning the reference's ``BuildOutcome``), its
``HarnessEvaluator`` and its ``cuda-single`` geometry resolver, on the reference's own
``tasks/rmsnorm``.  The reference then checks every identity it checks for Metal: the Track
selection, the rendered statement and ABI, the frozen geometry, the candidate digest in the build
provenance, the artifact-set digest in the report, and the schema-4 report reader.  The evaluator's
device run (``CudaTrackEvaluator.evaluate``, covered on the B200 by the GPU tests of the track
evaluator) is replaced here by a recorder, so these tests need no GPU; they do need the reference
checkout, which the GPU box does not have.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import pytest

REF = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))
ROOT = Path(__file__).resolve().parents[1]

RMSNORM = r'''#include <cuda_fp16.h>
extern "C" __global__ void rmsnorm(const __half* x, const __half* w, __half* y, long long M, long long H) {
    long long row = blockIdx.x;
    if (row >= M) return;
    __shared__ float part[256];
    float s = 0.f;
    for (long long i = threadIdx.x; i < H; i += blockDim.x) { float v = __half2float(x[row * H + i]); s += v * v; }
    part[threadIdx.x] = s;
    __syncthreads();
    for (int o = 128; o > 0; o >>= 1) { if (threadIdx.x < o) part[threadIdx.x] += part[threadIdx.x + o]; __syncthreads(); }
    float inv = rsqrtf(part[0] / (float)H + 1e-6f);
    for (long long i = threadIdx.x; i < H; i += blockDim.x) y[row * H + i] = __float2half(__half2float(x[row * H + i]) * inv * __half2float(w[i]));
}
/* taic-launch
kernel rmsnorm grid=M threads=256
*/
'''


@pytest.fixture(scope="module")
def seam():
    if not (REF / "tcenv").is_dir():
        pytest.skip("reference checkout not mounted")
    sys.path.append(str(REF))  # after this repository: the reference also has a `tests` package
    from shapeforge_b200 import bootstrap

    bootstrap.install()
    from tcenv.taskcontract import discover_standard_tasks
    from tcenv.taskcontract.runner import evaluate_task
    from tcenv.track import REPO_ROOT, CandidateArtifact, CandidateEntry

    locs = discover_standard_tasks(REF / "tasks", code_root=REPO_ROOT)
    loc = next(lc for lc in locs if lc.op_name == "rmsnorm" and lc.dtype == "fp16" and lc.size == "small")

    def candidate(source: str):
        return CandidateArtifact(track_id="cuda-single", entries=(
            CandidateEntry(path="kernel.cu", role="device_kernel", media_type="text/plain", data=source.encode()),))

    return evaluate_task, loc, candidate


def _run(seam, source, device_status="ok"):
    from shapeforge_b200 import harness_seam

    evaluate_task, loc, candidate = seam
    seen = []

    def device_run(req):
        seen.append(req)
        ok = device_status == "ok"
        return {"status": device_status, "cases": [{"case": c[0], "ok": ok} for c in req.cases[:1 if not ok else None]],
                "build": req.build.document(), "detail": "" if ok else "planted mismatch"}

    builder = harness_seam.HarnessBuilder()
    evaluator = harness_seam.HarnessEvaluator(run=device_run, cases=["normal", "large"])
    cand = candidate(source)
    result = evaluate_task(loc, track_id="cuda-single", candidate=cand, builder=builder, evaluator=evaluator,
                           geometry_resolver=harness_seam.geometry_resolver(loc),
                           track_registry_path=ROOT / "backends" / "cuda-sm100" / "tracks.json", target_id="b200")
    return result, seen, cand


def test_evaluate_task_runs_the_cuda_track_through_the_reference_pipeline(seam):
    import numpy as np
    import torch

    from shapeforge_b200.track_factory import CudaBuild

    result, seen, cand = _run(seam, RMSNORM)
    doc = result.document()
    assert doc["track"]["track_id"] == "cuda-single" and doc["candidate_sha256"] == cand.candidate_sha256
    rep = result.report
    assert rep["status"] == "ok" and rep["backend"] == "cuda-sm100" and rep["correctness"]["passed"] is True
    # The build record is the reference's projection of this builder's outcome: source, cubin and
    # the frozen geometry the reference attached, under the digest the reference re-checked.
    paths = {e["path"]: e["role"] for e in rep["build"]["artifacts"]["entries"]}
    assert paths == {"kernel.cu": "SOURCE", "kernel.cubin": "EXECUTABLE_MODULE", "execution_geometry.json": "AUXILIARY"}
    assert rep["build"]["artifacts"]["artifact_set_digest"] == result.artifact_set_digest
    assert rep["build"]["provenance"]["source_sha256"] == cand.candidate_sha256
    # The device run got the task's own request: the rmsnorm ABI at the small size, the task's
    # seeded cases with their fp64 references, its tolerances, and the nvcc build.
    (req,) = seen
    assert [(s.name, s.role) for s in req.specs] == [("x", "input"), ("w", "input"), ("y", "output")]
    m, h = req.specs[0].shape
    assert [c[0] for c in req.cases] == ["normal", "large"]
    x, w = (req.cases[0][1][n].double().numpy() for n in ("x", "w"))
    np.testing.assert_allclose(req.cases[0][2]["y"], x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * w, rtol=1e-12)
    assert (req.rtol, req.atol_rel) == (0.002, 0.001) and req.cases[0][1]["x"].dtype == torch.float16
    assert isinstance(req.build, CudaBuild) and req.build.kernels == ("rmsnorm",) and len(req.build.image) > 0
    # The geometry the reference froze is the launch block evaluated at this size.
    geo = result.document()["geometry_identity"]
    assert geo and req.build.stages[0].resolve({"M": m, "H": h}).grid[0] == m


def test_a_failing_device_run_is_reported_with_the_reference_status(seam):
    result, _, _ = _run(seam, RMSNORM, device_status="incorrect")
    rep = result.report
    assert rep["status"] == "incorrect" and rep["stage"] == "correctness" and rep["correctness"]["passed"] is False
    assert "planted mismatch" in rep["message"]


def test_a_candidate_without_a_launch_block_is_refused_before_any_build(seam):
    from tcenv.contract_errors import GeometryError

    with pytest.raises(GeometryError, match="taic-launch"):
        _run(seam, RMSNORM.split("/* taic-launch")[0])
