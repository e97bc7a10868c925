"""The reference's v2 evaluation seam, driven by this backend's builder and evaluator.

``tcenv.taskcontract.runner.evaluate_task`` (runner.py:553) selects the Track, derives the ABI
and the task statement, resolves the geometry, and then calls two injected services: the builder
(``build(request) -> BuildOutcome``, runner.py:725) and the evaluator (``evaluate(request) ->
schema-4 report``, runner.py:735), cross-checking the candidate digest, the artifact-set digest
and the report schema.  This module provides both services for the ``cuda-single`` Track:

* :class:`HarnessBuilder` compiles the candidate's single ``.cu`` entry for sm_100a
  (:class:`~shapeforge_b200.track_factory.CudaTrackBuilder`) and returns the reference's
  ``BuildOutcome`` (tcenv/remote/artifact_builder.py:527): the source (``SOURCE``) and the cubin
  (``EXECUTABLE_MODULE``) as the artifact set; a ``compute-pipeline`` native executable whose
  descriptor records the kernels, launch stages and cubin digest and whose handle is the build;
  the nvcc build profile; and the provenance bound to the candidate's digest.
* :class:`HarnessEvaluator` runs the task's correctness cases, and the timing when asked, on that
  build through :class:`~shapeforge_b200.track_factory.CudaTrackEvaluator`.  The request is
  read from the task directory the locator names (``eval_task.prepare``: the opspec's ABI, the
  task's own seeded inputs and fp64 reference, its tolerances).  It returns the reference's
  ``EvalReport`` (tcenv/evaluate.py:118) as a schema-4 document whose ``build`` is projected from
  the ``BuildOutcome`` (``project_full``).

Both import ``tcenv`` and exist for the harness process, which has it.  ``HarnessEvaluator(run=...)``
replaces the device run (the ``CudaTrackEvaluator.evaluate`` call) with a caller-supplied function
of the same signature; the host tests use it to drive the seam without a GPU.
"""

from __future__ import annotations

import hashlib
import subprocess
from typing import Any, Callable, Mapping, Sequence

from .track_factory import BACKEND_ID, CudaBuild, CudaTrackBuilder, CudaTrackEvaluator, EvaluationRequest, candidate_text

SOURCE_PATH = "kernel.cu"
CUBIN_PATH = "kernel.cubin"
BUILD_PROFILE_ID = "cuda-sm100-nvcc-v1"
BUILDER_ID = "cuda-sm100-nvcc"
BUILDER_VERSION = "1"


def _nvcc_version() -> str:
    from .build import nvcc

    try:
        out = subprocess.run([nvcc(), "--version"], capture_output=True, text=True, timeout=60).stdout
    except Exception:  # noqa: BLE001 - recorded as unknown, the build itself reports a missing nvcc
        return "unknown"
    lines = [ln for ln in out.splitlines() if "release" in ln]
    return lines[-1].split("release", 1)[1].strip()[:64] if lines else "unknown"


def build_profile(flags: Sequence[str]):
    """The reference's ``BuildProfile`` of this builder (toolchain nvcc, target sm_100a)."""
    from tcenv.remote.artifact_builder import BuildProfile

    return BuildProfile(
        build_profile=BUILD_PROFILE_ID,
        builder_id=BUILDER_ID,
        builder_version=BUILDER_VERSION,
        build_host="control_host",
        toolchain_id="nvcc",
        toolchain_version=_nvcc_version(),
        sdk_version="cuda",
        compile_profile={"language": "cuda", "arch": "sm_100a", "flags": " ".join(flags)},
    )


def geometry_resolver(locator: Any) -> Callable[[Any], Any]:
    """The ``cuda-single`` geometry resolver ``evaluate_task`` needs for a single-file Track
    (runner.py:445-459 refuses to invent one): the candidate's ``taic-launch`` block, each stage's
    grid / threads / shared memory evaluated with the symbols of the locator's task size (as the
    Metal single-source resolver does with its launch constants)."""
    from tcenv.contract_errors import GeometryError
    from tcenv.track.plane import ExecutionGeometry, GeometryStage

    from . import portfolio_pack as pp
    from .backend import parse_launch_templates

    opspec = pp.load_opspec(locator.task_dir)
    points = pp.domain(opspec, locator.dtype, [locator.size])
    if not points:
        raise GeometryError(f"size {locator.size!r} is not declared for {locator.dtype}")
    names = dict(points[0].names)

    def resolve(candidate: Any) -> Any:
        if not getattr(candidate, "single_source", False):
            raise GeometryError("the cuda-single resolver accepts exactly one device_kernel entry")
        try:
            templates = parse_launch_templates(candidate_text(candidate))
        except ValueError as exc:
            raise GeometryError(f"the cuda-single taic-launch block is invalid: {exc}") from exc
        if not templates:
            raise GeometryError("cuda-single needs one /* taic-launch */ block; the harness does not invent a grid or threads")
        stages = []
        for t in templates:
            r = t.resolve(names)
            stages.append(GeometryStage(kernel=r.kernel, grid=tuple(int(x) for x in r.grid), threads=tuple(int(x) for x in r.threads),
                                        threadgroup_bytes=int(r.smem)))
        return ExecutionGeometry(source="candidate", stages=tuple(stages))

    return resolve


class HarnessBuilder(CudaTrackBuilder):
    """``build(CandidateBuildRequest) -> BuildOutcome`` for the reference's ``evaluate_task``."""

    def build(self, request: Any, use_cache: bool = True) -> Any:  # noqa: D401 - the harness's builder interface
        from tcenv.remote.artifact_builder import BuildArtifact, BuildEvidence, BuildOutcome, BuildProvenance
        from tcenv.remote.artifact_bundle import ArtifactBundle, BundleEntry, NativeExecutable

        candidate = getattr(request, "candidate", None)
        if candidate is None:
            return super().build(request, use_cache=use_cache)
        built: CudaBuild = super().build(request, use_cache=use_cache)
        source = candidate_text(candidate).encode("utf-8")
        src_sha = hashlib.sha256(source).hexdigest()
        entries = (
            BundleEntry(path=SOURCE_PATH, role="SOURCE", media_type="text/plain", size_bytes=len(source), sha256=src_sha, data=source),
            BundleEntry(path=CUBIN_PATH, role="EXECUTABLE_MODULE", media_type="application/octet-stream", size_bytes=len(built.image),
                        sha256=built.image_sha256, data=built.image),
        )
        descriptor = {
            "backend": BACKEND_ID,
            "target": "sm_100a",
            "kernels": list(built.kernels),
            "cubin_sha256": built.image_sha256,
            "stages": [dict(d) for d in built.document()["stages"]],
        }
        native = NativeExecutable(backend_id=BACKEND_ID, kind="compute-pipeline", entry_path=SOURCE_PATH, entry_sha256=src_sha,
                                  descriptor=descriptor, handle=built)
        bundle = ArtifactBundle(entries=entries, native=native)
        provenance = BuildProvenance(profile=build_profile(built.flags), source_sha256=candidate.candidate_sha256,
                                     artifact_set_digest=bundle.artifact_set_digest)
        evidence = BuildEvidence(mode="prebuilt", status="ok", provenance=provenance,
                                 artifacts=tuple(BuildArtifact.from_entry(e) for e in bundle.entries), placement="control_host",
                                 native=native)
        return BuildOutcome(bundle=bundle, provenance=provenance, evidence=evidence)


# The report's status for each CudaTrackEvaluator status, and the stage it reached.
_STAGE = {"ok": "bench", "incorrect": "correctness", "unsafe": "correctness", "runtime_error": "correctness",
          "abi_error": "abi", "compile_error": "compile", "timeout": "correctness", "crash": "correctness"}


class HarnessEvaluator(CudaTrackEvaluator):
    """``evaluate(CandidateEvaluationRequest) -> schema-4 report`` for ``evaluate_task``.

    ``cases``: the task cases to run (default: every declared case); ``timed``: also time the
    candidate (the interleaved protocol, ``time_reps`` repetitions); ``run``: the device run
    (default ``CudaTrackEvaluator.evaluate``)."""

    def __init__(self, *, cases: Sequence[str] | None = None, timed: bool = False, time_reps: int = 15,
                 run: Callable[[EvaluationRequest], Mapping[str, Any]] | None = None) -> None:
        super().__init__(HarnessBuilder())
        self.cases = None if cases is None else list(cases)
        self.timed = timed
        self.time_reps = time_reps
        self._run = run
        self.last_device_report: Mapping[str, Any] | None = None

    def evaluate(self, request: Any) -> Any:  # noqa: D401 - the harness's evaluator interface
        if not hasattr(request, "build_request"):
            return super().evaluate(request)
        from tcenv.build_projection import project_full
        from tcenv.evaluate import EvalReport
        from tcenv.schema import PROTOCOL_VERSION

        from . import eval_task

        locator = request.build_request.locator
        contract = request.build_request.contract
        outcome = request.build
        native = outcome.bundle.native
        built = native.handle if native is not None and isinstance(native.handle, CudaBuild) else None
        prepared = eval_task.prepare(locator.task_dir, locator.dtype, locator.size, cases=self.cases)
        device_request = EvaluationRequest(
            specs=prepared["specs"], cases=prepared["cases"], rtol=prepared["rtol"], atol_rel=prepared["atol_rel"],
            exact=prepared["exact"], build=built, source=None if built is not None else candidate_text(request.build_request.candidate),
            scalars=prepared["scalars"], output_dtypes=prepared.get("output_dtypes", {}), names=prepared["names"],
            time_reps=self.time_reps if self.timed else 0)
        result = dict((self._run or super().evaluate)(device_request))
        self.last_device_report = result
        status = str(result.get("status", "crash"))
        passed = status == "ok"
        identity = {"opspec_digest": contract.spec.digest, "lowering_profile_digest": contract.fingerprint()}
        timing = result.get("timing") or {}
        cand = timing.get("candidate") or {}
        report = EvalReport(
            task=locator.op_name,
            dtype=locator.dtype,
            size=locator.size,
            mode="timed" if self.timed else "correctness",
            status=status,
            stage=_STAGE.get(status, "correctness"),
            message=str(result.get("detail", ""))[:2000],
            seed=eval_task.SEARCH_SEED,
            correctness={"passed": passed, "cases": list(result.get("cases", []))},
            pipeline=dict(result.get("pipeline") or {}),
            benchmark={"protocol": timing.get("protocol"), "noise_cv": timing.get("noise_cv"), "attempts": timing.get("attempts"),
                       "candidate": cand} if timing else {},
            candidate_us=(float(cand["median_s"]) * 1e6) if cand.get("median_s") is not None else None,
            build=project_full(outcome, build_kind="native", identity=identity),
            protocol_version=PROTOCOL_VERSION,
            target_id=request.build_request.target_id,
            backend=BACKEND_ID,
            backend_version="1",
        )
        return report.to_json()
