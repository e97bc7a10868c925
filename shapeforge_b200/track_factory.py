"""Fail-closed construction of the cuda-sm100 Track adapters.

The reference's v2 worker resolves a candidate's build and evaluation services through
``Backend.track_adapter(spec)`` (tcenv/backends/metal/backend.py:39-43 ->
tcenv/backends/metal/track_factory.py:139-196).  This module is the CUDA counterpart for the
``cuda-single`` Track of ``backends/cuda-sm100/tracks.json``: a single ``.cu`` source whose
``extern "C" __global__`` kernels take the task's ABI tensors in order, with a ``taic-launch``
block naming the stages.  Only that registered identity (renderer / validator / build ids and
versions, delivery ``single_source``) is accepted; any other identity is refused, never routed
to a different adapter.

Services (resolved lazily, each constructed once per adapter):

* ``builder``   -> :class:`CudaTrackBuilder`: ``prepare`` runs the pre-compile checks (screen,
  launch block, kernel names present); ``build`` compiles for sm_100a with nvcc to a cubin;
* ``evaluator`` -> :class:`CudaTrackEvaluator`: loads the cubin through the C ABI and runs the
  three guarded correctness trials per case (``runtime.CorrectnessRunner``) and, when asked, the
  interleaved timing protocol (``protocol.measure_interleaved``);
* ``renderer``  -> the ABI stub of a contract (``CudaBackend.abi_stub``);
* ``validator`` -> a callable returning the refusal list of a source (empty = accepted).
"""

from __future__ import annotations

import hashlib
import re
from dataclasses import dataclass, field
from typing import Any, Callable, Mapping, Sequence

BACKEND_ID = "cuda-sm100"
SINGLE = (
    "cuda-sm100.track.cuda-single.renderer",
    1,
    "cuda-sm100.track.cuda-single.validator",
    1,
    "cuda-sm100.track.cuda-single.build",
    1,
    "single_source",
)


class TrackRefused(ValueError):
    """The Track identity or the candidate is not one this backend implements."""


def _unsupported(message: str) -> Exception:
    """The reference's typed refusal when tcenv is importable (the harness process), else ours."""
    try:
        from tcenv.contract_errors import UnsupportedContractCapability

        return UnsupportedContractCapability(message)
    except Exception:  # noqa: BLE001 - tcenv is optional outside the harness
        return TrackRefused(message)


def implementation_tuple(spec: Any) -> tuple:
    return (
        spec.renderer.implementation_id,
        spec.renderer.implementation_version,
        spec.validator.implementation_id,
        spec.validator.implementation_version,
        spec.build_adapter.implementation_id,
        spec.build_adapter.implementation_version,
        spec.delivery,
    )


def profile(spec: Any) -> str:
    """``"cuda-single"`` for the registered identity; refuse anything else."""
    identity = implementation_tuple(spec)
    if identity == SINGLE and int(spec.track_version) == 1:
        return "cuda-single"
    raise _unsupported(f"no CUDA adapter implements the registered identity {identity!r} for "
                       f"{spec.track_id}/{spec.track_version}")


# ---- candidate text ----------------------------------------------------------------------------


def candidate_text(candidate: Any) -> str:
    """Source text of a single-source candidate: a ``str``, ``bytes``, or the reference's
    ``CandidateArtifact`` (tcenv/track/plane.py:388) with exactly one ``device_kernel`` entry."""
    if isinstance(candidate, str):
        return candidate
    if isinstance(candidate, (bytes, bytearray)):
        return bytes(candidate).decode("utf-8")
    entries = getattr(candidate, "entries", None)
    if entries is None:
        raise TrackRefused(f"cannot read a candidate source from {type(candidate).__name__}")
    if len(entries) != 1 or getattr(entries[0], "role", "device_kernel") != "device_kernel":
        raise TrackRefused("the cuda-single track takes exactly one device_kernel entry")
    data = entries[0].data
    return data.decode("utf-8") if isinstance(data, (bytes, bytearray)) else str(data)


@dataclass(frozen=True)
class CudaBuild:
    """One successful build: the cubin image and its provenance."""

    source_sha256: str
    image_sha256: str
    image: bytes
    kernels: tuple[str, ...]
    stages: tuple[Any, ...]
    flags: tuple[str, ...]
    cache_hit: bool = False  # the image came from the cubin cache rather than from an nvcc run
    resources: Mapping[str, Any] = field(default_factory=dict)  # entry -> kernel_stats.KernelResources

    def document(self) -> dict[str, Any]:
        return {
            "source_sha256": self.source_sha256,
            "image_sha256": self.image_sha256,
            "image_bytes": len(self.image),
            "kernels": list(self.kernels),
            "stages": [_stage_document(s) for s in self.stages],
            "symbolic_launch": any(s.symbolic for s in self.stages),
            "flags": list(self.flags),
            "target": "sm_100a",
            "cache_hit": self.cache_hit,
        }


def _stage_document(stage: Any) -> dict[str, Any]:
    """A launch stage for the build record: integers when literal, the expressions otherwise."""
    if not stage.symbolic:
        r = stage.resolve({})
        return {"kernel": r.kernel, "grid": list(r.grid), "threads": list(r.threads), "smem": r.smem}
    return {"kernel": stage.kernel, "grid": list(stage.grid), "threads": list(stage.threads), "smem": stage.smem}


class CudaTrackBuilder:
    """Pre-compile checks and the nvcc build of a cuda-single candidate."""

    build_kind = "native"

    def __init__(self, *, target_id: str = "b200", extra_flags: Sequence[str] = ()) -> None:
        from .backend import CudaBackend

        self.target_id = target_id
        self.extra_flags = tuple(extra_flags)
        self._backend = CudaBackend()

    def _request_source(self, request: Any) -> str:
        cand = getattr(request, "candidate", request)
        return candidate_text(cand)

    def check(self, source: str) -> tuple:
        """Screen + launch block; return the launch templates (values may be expressions over the
        task's symbols, resolved per shape at launch) or raise :class:`TrackRefused`."""
        from .backend import parse_launch_templates

        problems = self._backend.screen(source)
        if problems:
            raise TrackRefused("candidate refused before compilation: " + "; ".join(problems))
        try:
            stages = parse_launch_templates(source)
        except ValueError as exc:
            raise TrackRefused(f"launch block: {exc}") from exc
        if not stages:
            raise TrackRefused("the candidate has no taic-launch block")
        for st in stages:
            if not re.search(self._backend.source_name_pattern(st.kernel), source):
                raise TrackRefused(f"launch stage kernel {st.kernel!r} is not an extern \"C\" __global__ kernel of the source")
        return tuple(stages)

    def prepare(self, request: Any) -> None:
        """Every check that needs no compiler and no device."""
        self.check(self._request_source(request))

    def build(self, request: Any, use_cache: bool = True) -> CudaBuild:
        """Compile once for sm_100a; a compiler failure raises ``CudaCompileError`` with the log.
        ``use_cache=False`` forces nvcc to run (``CudaBuild.cache_hit`` is then False)."""
        from .backend import CudaCompileError
        from .candidates import CandidateCompileError, compile_source

        source = self._request_source(request)
        stages = self.check(source)
        flags = ("-lineinfo",) + self.extra_flags
        try:
            from .candidates import cache_path, kernel_resources

            cache_hit = use_cache and cache_path(source, flags, "track").is_file()
            image = compile_source(source, extra_flags=flags, name="track", use_cache=use_cache)
            resources = kernel_resources(source, flags, "track")
        except CandidateCompileError as exc:
            raise CudaCompileError(f"{exc}\n{exc.log}") from exc
        kernels = tuple(dict.fromkeys(s.kernel for s in stages))
        return CudaBuild(
            source_sha256=hashlib.sha256(source.encode()).hexdigest(),
            image_sha256=hashlib.sha256(image).hexdigest(),
            image=image,
            kernels=kernels,
            stages=stages,
            flags=flags,
            cache_hit=cache_hit,
            resources=resources,
        )


# ---- evaluation --------------------------------------------------------------------------------


@dataclass
class EvaluationRequest:
    """What one evaluation needs when the caller is not the reference's v2 worker: the source
    (or a finished :class:`CudaBuild`), the ABI tensors in order, the correctness cases
    ``(name, inputs, refs, scales)`` and the task tolerances; ``scalars`` are extra kernel
    arguments (ctypes values) appended after the tensor pointers."""

    specs: Sequence[Any]
    cases: Sequence[tuple]
    rtol: float
    atol_rel: float
    exact: bool = False
    source: str | None = None
    build: CudaBuild | None = None
    scalars: Sequence[Any] = ()
    output_dtypes: Mapping[str, str] = field(default_factory=dict)
    time_reps: int = 0
    names: Mapping[str, int] = field(default_factory=dict)  # the shape's symbols, for symbolic launch values


class CudaTrackEvaluator:
    """Correctness (three guarded trials per case) and optional timing of a built candidate."""

    def __init__(self, builder: CudaTrackBuilder | None = None) -> None:
        self.builder = builder or CudaTrackBuilder()

    @staticmethod
    def launcher(build: CudaBuild, scalars: Sequence[Any] = (), stream: int | None = None,
                 names: Mapping[str, int] | None = None) -> Callable[[list[int]], None]:
        """``launch(pointers)`` running every stage of the build in order on the current stream;
        ``names`` (the shape's symbols) resolve symbolic launch values once, here."""
        import torch

        from .candidates import Module

        stages = [st.resolve(names) for st in build.stages]
        module = Module(build.image)

        def launch(ptrs: list[int]) -> None:
            s = torch.cuda.current_stream().cuda_stream if stream is None else stream
            for st in stages:
                module.launch(st.kernel, st.grid, st.threads, list(ptrs) + list(scalars), smem=st.smem, stream=s)

        launch.module = module  # keep the image loaded as long as the launcher lives
        return launch

    def evaluate(self, request: EvaluationRequest) -> dict[str, Any]:
        from .backend import CudaCompileError

        report: dict[str, Any] = {"backend": BACKEND_ID, "track": "cuda-single"}
        try:
            build = request.build or self.builder.build(request.source)
        except TrackRefused as exc:
            return dict(report, status="unsafe", detail=str(exc))
        except CudaCompileError as exc:
            return dict(report, status="compile_error", detail=str(exc))
        report["build"] = build.document()
        if build.resources:
            # Compiled resources against the launch, before anything launches (Backend.check_abi).
            from . import kernel_stats

            try:
                stages = [st.resolve(request.names) for st in build.stages]
            except Exception:  # noqa: BLE001 - the launcher below reports an unresolvable launch
                stages = []
            problems = kernel_stats.check_stages(build.resources, stages)
            if problems:
                return dict(report, status="abi_error", detail="; ".join(problems))
            if stages:
                report["pipeline"] = kernel_stats.stats_many([(build.resources[s.kernel], s) for s in stages])
        try:
            launch = self.launcher(build, request.scalars, names=request.names)
            from .runtime import CorrectnessRunner

            from .gpulock import gpu_lock

            runner = CorrectnessRunner(request.specs, launch, output_dtypes=request.output_dtypes)
            results = []
            from .heartbeat import launching

            with gpu_lock("correctness", exclusive=False):  # untimed: may overlap other untimed work, never a timing
                for name, inputs, refs, scales in request.cases:
                    with launching():  # the launch deadline covers each case's three trials
                        res = runner.run_case(name, inputs, refs, scales, request.rtol, request.atol_rel, request.exact)
                    results.append(res)
                    if not res.ok:
                        break
        except Exception as exc:  # noqa: BLE001 - a device error is the candidate's runtime_error
            return dict(report, status="runtime_error", detail=str(exc))
        report["cases"] = [r.summary() for r in results]
        bad = next((r for r in results if not r.ok), None)
        if bad is not None:
            report["status"] = "unsafe" if bad.safety else "incorrect"
            return report
        report["status"] = "ok"
        if request.time_reps > 0:
            report["timing"] = self._time(launch, runner, request.time_reps)
        return report

    @staticmethod
    def _time(launch, runner, reps: int) -> dict[str, Any]:
        """The reference's interleaved protocol (median of ``reps`` batches, CV gate, attempts)."""
        from . import protocol

        from .gpulock import gpu_lock

        from .heartbeat import launching

        ptrs = runner.pointers()
        batch = protocol.cuda_event_runner(lambda i: launch(ptrs))

        def run_k(k: int) -> float:
            with launching():  # one synchronised k-launch batch
                return batch(k)

        with gpu_lock("candidate timing"):  # exclusive on this GPU for the whole measurement
            noise, stats, attempts = protocol.measure_interleaved({"candidate": run_k}, reps=reps)
        return {"protocol": "interleaved", "noise_cv": noise, "attempts": attempts, "candidate": stats["candidate"].to_dict()}


def adapter_for_track(spec: Any):
    """Resolve the registered implementation for ``spec`` (a TrackSpec) without reading a
    default registry.  Returns the reference's ``LazyTrackAdapter`` when tcenv is importable,
    else an equivalent local object with the same ``resolve(service)`` contract."""
    profile(spec)
    factories: dict[str, Callable[[], Any]] = {
        "builder": lambda: CudaTrackBuilder,
        "evaluator": lambda: CudaTrackEvaluator,
        "renderer": lambda: _renderer,
        "validator": lambda: _validator,
    }
    try:
        from tcenv.track.adapter import LazyTrackAdapter

        return LazyTrackAdapter(spec, factories)
    except Exception:  # noqa: BLE001
        return _LocalAdapter(spec, factories)


def _renderer(contract: Any) -> str:
    from .backend import CudaBackend

    return CudaBackend().abi_stub(contract)


def _validator(candidate: Any) -> list[str]:
    try:
        CudaTrackBuilder().check(candidate_text(candidate))
    except TrackRefused as exc:
        return [str(exc)]
    return []


@dataclass
class _LocalAdapter:
    spec: Any
    _factories: Mapping[str, Callable[[], Any]]
    _resolved: dict[str, Any] = field(default_factory=dict)

    def resolve(self, service: str) -> Any:
        if service in self._resolved:
            return self._resolved[service]
        factory = self._factories.get(service)
        if factory is None:
            raise _unsupported(f"track {self.spec.track_id}/{self.spec.track_version} has no registered {service!r} adapter binding")
        self._resolved[service] = factory()
        return self._resolved[service]


__all__ = ["adapter_for_track", "CudaTrackBuilder", "CudaTrackEvaluator", "CudaBuild", "EvaluationRequest", "TrackRefused",
           "SINGLE", "profile"]
