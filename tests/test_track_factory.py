"""The cuda-single Track plug-in: fail-closed identity resolution, pre-compile checks, the nvcc
build, and (on a B200) the guarded correctness trials + timing of a compiled candidate.

The reference resolves Track services through ``Backend.track_adapter(spec)``
(tcenv/backends/metal/track_factory.py:139-196); the spec here is loaded from
``backends/cuda-sm100/tracks.json`` with the reference's own registry loader when the reference
is mounted, else built from the same document.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest

from shapeforge_b200 import track_factory as tf
from shapeforge_b200.backend import CudaBackend, CudaCompileError

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))

SILU = r'''
#include <cuda_fp16.h>
/* taic-launch
kernel silu_candidate grid=64,1,1 threads=256,1,1
*/
extern "C" __global__ void __launch_bounds__(256) silu_candidate(const __half* __restrict__ x, __half* __restrict__ y) {
    const int i = blockIdx.x * 256 + threadIdx.x;
    const float v = __half2float(x[i]);
    y[i] = __float2half_rn(v / (1.0f + expf(-v)));
}
'''

WRONG = SILU.replace("v / (1.0f + expf(-v))", "v")


def _spec():
    doc = json.loads((ROOT / "backends" / "cuda-sm100" / "tracks.json").read_text())["tracks"][0]
    if REF.is_dir():
        sys.path.append(str(REF))  # after this repository: the reference also has a `tests` package
        from tcenv.track.registry import load_track_registry

        reg = load_track_registry(ROOT / "backends" / "cuda-sm100" / "tracks.json")
        return next(t for t in reg.tracks if t.track_id == "cuda-single")
    part = lambda d: SimpleNamespace(**d)  # noqa: E731
    return SimpleNamespace(track_id=doc["track_id"], track_version=doc["track_version"], delivery=doc["delivery"],
                           renderer=part(doc["renderer"]), validator=part(doc["validator"]), build_adapter=part(doc["build_adapter"]))


def test_registered_identity_resolves_every_service():
    spec = _spec()
    assert tf.profile(spec) == "cuda-single"
    adapter = CudaBackend().track_adapter(spec)
    assert adapter.resolve("builder") is tf.CudaTrackBuilder
    assert adapter.resolve("evaluator") is tf.CudaTrackEvaluator
    assert adapter.resolve("validator")(SILU) == []
    assert adapter.resolve("validator")("__global__ void k() { __trap(); }")
    stub = adapter.resolve("renderer")({"tensors": [{"name": "x", "dtype": "fp16", "access": "read"},
                                                   {"name": "y", "dtype": "fp16", "access": "write"}]})
    assert stub.startswith('extern "C" __global__ void candidate(const __half* __restrict__ x, __half* __restrict__ y')
    with pytest.raises(Exception) as exc:
        adapter.resolve("confirmation")
    assert "no registered" in str(exc.value)


def test_other_identities_are_refused():
    spec = _spec()
    bad = SimpleNamespace(track_id="cuda-single", track_version=1, delivery="candidate_bundle",
                          renderer=spec.renderer, validator=spec.validator, build_adapter=spec.build_adapter)
    with pytest.raises(Exception, match="no CUDA adapter"):
        tf.adapter_for_track(bad)
    v2 = SimpleNamespace(track_id="cuda-single", track_version=2, delivery=spec.delivery,
                         renderer=spec.renderer, validator=spec.validator, build_adapter=spec.build_adapter)
    with pytest.raises(Exception, match="no CUDA adapter"):
        tf.profile(v2)


def test_prepare_refuses_before_the_compiler():
    b = tf.CudaTrackBuilder()
    b.prepare(SILU)
    for src, why in ((SILU.replace("/* taic-launch", "/* no-launch"), "no taic-launch"),
                     (SILU.replace("kernel silu_candidate", "kernel other_name"), "is not an extern"),
                     (SILU + "\n__device__ void f() { __trap(); }\n", "trap"),
                     (SILU.replace("grid=64,1,1", "grid=ceil_div(64)"), "launch block"),
                     (SILU.replace("grid=64,1,1", "grid=eq(N,1)"), "launch block")):
        with pytest.raises(tf.TrackRefused, match=why):
            b.prepare(src)
    with pytest.raises(tf.TrackRefused, match="exactly one device_kernel"):
        b.prepare(SimpleNamespace(candidate=SimpleNamespace(entries=())))


def test_symbolic_launch_values_resolve_per_shape():
    """Launch values may be expressions over the task's symbols (the portfolio geometry
    language); they are checked at prepare and resolved per shape at launch."""
    from shapeforge_b200.backend import parse_launch_templates

    src = SILU.replace("grid=64,1,1", "grid=ceil_div(N,256)")
    tf.CudaTrackBuilder().prepare(src)
    (tpl,) = parse_launch_templates(src)
    assert tpl.symbolic
    assert tpl.resolve({"N": 16384}).grid == (64, 1, 1)
    assert tpl.resolve({"N": 16385}).grid == (65, 1, 1)
    with pytest.raises(Exception, match="not declared"):
        tpl.resolve({})


def test_reference_candidate_artifact_is_read():
    entry = SimpleNamespace(role="device_kernel", data=SILU.encode(), path="k.cu")
    assert tf.candidate_text(SimpleNamespace(entries=(entry,))) == SILU


def test_build_compiles_for_sm100a():
    build = tf.CudaTrackBuilder().build(SILU)
    assert build.kernels == ("silu_candidate",) and len(build.image) > 1000
    doc = build.document()
    assert doc["target"] == "sm_100a" and doc["stages"][0]["grid"] == [64, 1, 1]
    with pytest.raises(CudaCompileError):
        tf.CudaTrackBuilder().build(SILU.replace("expf(-v)", "expf(-v"))


def _silu_case(dev_n=64 * 256):
    import torch

    from oracle import ops as oref
    from shapeforge_b200 import cases, compare
    from shapeforge_b200.runtime import TensorSpec

    x = cases.sample("normal", (dev_n,), 11, "fp16").to(torch.float16)
    ref = oref.silu(x.double().numpy())
    specs = [TensorSpec("x", (dev_n,), torch.float16, "input"), TensorSpec("y", (dev_n,), torch.float16, "output")]
    return specs, [("normal", {"x": x}, {"y": ref}, {"y": compare.rms_scale(ref)})]


@pytest.mark.gpu
def test_evaluator_runs_the_guarded_trials_and_times(cuda_device):
    specs, case = _silu_case()
    ev = tf.CudaTrackEvaluator()
    rep = ev.evaluate(tf.EvaluationRequest(specs=specs, cases=case, rtol=2e-3, atol_rel=1e-3, source=SILU, time_reps=3))
    assert rep["status"] == "ok", rep
    assert rep["timing"]["candidate"]["median_s"] > 0
    bad = ev.evaluate(tf.EvaluationRequest(specs=specs, cases=case, rtol=2e-3, atol_rel=1e-3, source=WRONG))
    assert bad["status"] == "incorrect", bad
    assert ev.evaluate(tf.EvaluationRequest(specs=specs, cases=case, rtol=2e-3, atol_rel=1e-3,
                                            source=SILU.replace("expf(-v)", "expf(-v")))["status"] == "compile_error"
