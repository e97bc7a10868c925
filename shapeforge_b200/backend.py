"""``CudaBackend``: the B200 implementation of the harness's Backend protocol.

The reference's evaluation layer talks to an accelerator only through
``tcenv.backends.base.Backend`` (tcenv/backends/base.py:75-455), loaded from
``backends/<id>/backend.toml`` by ``tcenv.backends.registry.load_backend``
(tcenv/backends/registry.py:34-76).  This class fills that protocol for CUDA sm_100a:

* parent-process (text-only) hooks — ``screen``, ``parse_launch``, ``validate_launch``,
  ``device_matches``, ``limit_notes``, ``calibration``, ``roofline``, ``describe`` ... — never touch
  the device;
* child-process hooks — ``context``, ``probe``, ``run_correctness``, ``prepare_bench`` — run the
  C-ABI library (``shapeforge_b200._native``) and the guarded-buffer runtime.

``roofline`` restates tcenv/backends/metal/profile.py:251-283 (the memory time of the task's
minimum bytes against the copy bandwidth, the compute time of its flops against the dense peak,
bound = the larger) with the B200 calibration of ``targets/b200/calibration.json`` or the pool's
measured peaks.
"""

from __future__ import annotations

import json
import re
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Mapping

ROOT = Path(__file__).resolve().parent.parent
BACKEND_ID = "cuda-sm100"
BACKEND_VERSION = "1"

# A candidate's bulk copy with the cluster-multicast qualifier (the qualifier is spelled out in
# two pieces so that this source names no such copy itself).
_CLUSTER_MULTICAST = re.compile("multi" + r"cast\s*::\s*cluster")


@dataclass(frozen=True)
class DeviceInfo:
    """Field-for-field the reference's ``DeviceInfo`` (tcenv/backends/base.py:31-47)."""

    backend: str
    name: str
    family: str
    limits: Mapping[str, Any] = field(default_factory=dict)
    raw: Mapping[str, Any] = field(default_factory=dict)
    matches: bool = False
    match_error: str = ""
    warnings: tuple[str, ...] = ()


@dataclass(frozen=True)
class Capabilities:
    supports_launch_spec: bool = True
    supports_validation: bool = False
    supports_device_timestamps: bool = True
    supports_profiler: bool = True
    supports_hw_features: bool = True
    supports_feature_signature: bool = False


class CudaRuntimeError(RuntimeError):
    """A device-side failure reported by the C ABI (status 3) or a bounded wait that gave up."""


class CudaCompileError(RuntimeError):
    """A candidate source that nvcc rejected."""


# The launch block a CUDA candidate carries, like the MSL `/* taic-launch ... */` block
# (tcenv/backends/metal/launch.py:1-60): `kernel <name> grid=X[,Y[,Z]] threads=X[,Y[,Z]] [smem=B]`.
# Each value is an integer or an expression over the task's symbols in the guard/geometry language
# of ``expr`` (``grid=ceil_div(N,256)``), so one source can serve every shape a portfolio variant
# covers; the expressions are resolved per shape (``LaunchTemplate.resolve``).
_LAUNCH_BLOCK = re.compile(r"/\*\s*taic-launch(.*?)\*/", re.S)
_LAUNCH_LINE = re.compile(r"^\s*kernel\s+(\w+)\s+grid=(.+?)\s+threads=(.+?)(?:\s+smem=(.+?))?\s*$")
MAX_STAGES = 32


@dataclass(frozen=True)
class LaunchStage:
    kernel: str
    grid: tuple[int, int, int]
    threads: tuple[int, int, int]
    smem: int = 0


def _split_top(text: str) -> list[str]:
    """Split a launch value at commas outside parentheses."""
    parts, depth, cur = [], 0, ""
    for ch in text:
        if ch == "," and depth == 0:
            parts.append(cur)
            cur = ""
            continue
        depth += ch == "("
        depth -= ch == ")"
        cur += ch
    parts.append(cur)
    return [p.strip() for p in parts]


@dataclass(frozen=True)
class LaunchTemplate:
    """One launch line with its values kept as expressions (text) until a shape is known."""

    kernel: str
    grid: tuple[str, ...]
    threads: tuple[str, ...]
    smem: str = "0"

    @property
    def symbolic(self) -> bool:
        from . import expr

        return any(expr.names(expr.parse(t)) for t in (*self.grid, *self.threads, self.smem))

    def resolve(self, names: Mapping[str, int] | None = None) -> LaunchStage:
        from . import expr

        env = dict(names or {})

        def dims(terms: tuple[str, ...], what: str) -> tuple[int, int, int]:
            vals = [int(expr.evaluate_term(t, env, where=f"{self.kernel} {what}")) for t in terms]
            if any(v < 1 for v in vals):
                raise ValueError(f"{self.kernel}: {what} {vals} has a dimension below 1")
            return tuple(vals + [1] * (3 - len(vals)))  # type: ignore[return-value]

        smem = int(expr.evaluate_term(self.smem, env, where=f"{self.kernel} smem"))
        if smem < 0:
            raise ValueError(f"{self.kernel}: negative shared memory")
        return LaunchStage(self.kernel, dims(self.grid, "grid"), dims(self.threads, "threads"), smem)


def parse_launch_templates(source: str) -> list[LaunchTemplate] | None:
    """The launch block of ``source`` as templates (None without a block); syntax is checked,
    names are not resolved."""
    from . import expr

    m = _LAUNCH_BLOCK.search(source)
    if not m:
        return None
    out = []
    for line in m.group(1).splitlines():
        if not line.strip():
            continue
        lm = _LAUNCH_LINE.match(line)
        if not lm:
            raise ValueError(f"unparseable launch line {line.strip()!r}")
        grid, threads = _split_top(lm.group(2)), _split_top(lm.group(3))
        if not 1 <= len(grid) <= 3 or not 1 <= len(threads) <= 3:
            raise ValueError(f"bad launch dimensions in {line.strip()!r}")
        tpl = LaunchTemplate(lm.group(1), tuple(grid), tuple(threads), (lm.group(4) or "0").strip())
        for t in (*tpl.grid, *tpl.threads, tpl.smem):
            try:
                node = expr.parse(t, f"launch {tpl.kernel}")
                if expr.kind(node) != expr.INT:
                    raise ValueError(f"launch value {t!r} is a predicate")
            except expr.ExprError as exc:
                raise ValueError(str(exc)) from exc
        out.append(tpl)
    if not out or len(out) > MAX_STAGES:
        raise ValueError(f"a launch block needs 1..{MAX_STAGES} stages")
    return out


class CudaBackend:
    id = BACKEND_ID
    version = BACKEND_VERSION
    language = "cuda"
    file_ext = ".cu"
    display_name = "CUDA sm_100a (B200)"
    source_fence = "cuda"
    reference_skill = ""
    skill_names: tuple[str, ...] = ()
    skill_optimization = ""
    skill_profiling = ""
    skill_profiler = "ncu"
    skill_hardware = ""
    runtime_headers = "#include <cuda_fp16.h>\n#include <cuda_bf16.h>\n"
    capabilities = Capabilities()

    # ---- parent-process, text-only hooks -------------------------------------------------------

    def track_adapter(self, track):
        """Construct the adapter for an already-selected TrackSpec, lazily and fail-closed."""
        from .track_factory import adapter_for_track

        return adapter_for_track(track)

    def screen(self, source: str, task: Any = None) -> list[str]:
        """Static refusals before any build: forbidden constructs on this pool."""
        problems = []
        if re.search(r"\b__trap\s*\(|\basm\s*\(\s*\"trap", source):
            problems.append("trap is not allowed: report failures through a status word")
        if re.search(_CLUSTER_MULTICAST, source):
            problems.append("cluster-multicast bulk copies are not allowed on this backend")
        if "__global__" not in source:
            problems.append("no __global__ kernel in the candidate")
        return problems

    def parse_launch(self, source: str, contract: Any = None, names: Mapping[str, int] | None = None) -> list[LaunchStage] | None:
        """The launch stages resolved on ``names`` (the shape's symbols; a symbolic value without
        them is an error)."""
        from . import expr

        templates = parse_launch_templates(source)
        if templates is None:
            return None
        try:
            return [t.resolve(names) for t in templates]
        except expr.ExprError as exc:
            raise ValueError(str(exc)) from exc

    def source_name_pattern(self, kernel_name: str) -> str:
        return r'extern\s+"C"\s+__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s+)?' + re.escape(kernel_name) + r"\s*\("

    def launch_stage_count(self, source: str, contract: Any = None) -> int:
        stages = self.parse_launch(source, contract)
        return len(stages) if stages else 1

    def validate_launch(self, stages: list[LaunchStage], limits: Mapping[str, int]) -> list[str]:
        problems = []
        for st in stages:
            threads = st.threads[0] * st.threads[1] * st.threads[2]
            if threads > int(limits.get("max_threads_per_threadgroup", 1024)):
                problems.append(f"{st.kernel}: {threads} threads per CTA exceeds the limit")
            if st.smem > int(limits.get("max_threadgroup_memory_bytes", 232448)):
                problems.append(f"{st.kernel}: {st.smem} bytes of shared memory exceeds the limit")
            if st.grid[1] > 65535 or st.grid[2] > 65535:
                problems.append(f"{st.kernel}: grid y/z above 65535")
        return problems

    def validation_env(self, base_env: Mapping[str, str]) -> dict[str, str]:
        return dict(base_env)

    def worker_env(self, base_env: Mapping[str, str], *, validation: bool) -> dict[str, str]:
        return dict(base_env)

    def parse_validation_stderr(self, stderr: str) -> list[str]:
        return []

    def device_matches(self, target: Any, info: Mapping[str, Any]) -> bool:
        want = getattr(target, "match_name_contains", None) or (target or {}).get("match_name_contains", "B200")
        name = str(info.get("name", ""))
        major = int(info.get("cc_major", 10))
        return want in name and major == 10

    def limit_notes(self, target: Any, info: Mapping[str, Any]) -> list[str]:
        notes = []
        limits = getattr(target, "raw_limits", None) or {}
        live_smem = int(info.get("max_smem_per_block_optin", 0) or 0)
        declared = int(limits.get("max_threadgroup_memory_bytes", 0) or 0)
        if live_smem and declared and live_smem < declared:
            notes.append(f"device allows {live_smem} bytes of shared memory per CTA, target declares {declared}")
        return notes

    def calibration(self, target_id: str = "b200") -> dict:
        """Peak bandwidth / flops of the target: the pool's measured peaks when present, else the
        target's calibration.json (tcenv/target.py:194-204 keeps the same override order)."""
        peaks = ROOT / "MEASURED_PEAKS.json"
        if peaks.is_file():
            d = json.loads(peaks.read_text())
            return {
                "device": d.get("gpu_name", "NVIDIA B200"),
                "copy_gbs": float(d["hbm_gbs"]),
                "read_gbs": float(d["hbm_gbs"]),
                "peak_tflops": {"fp16": float(d["bf16_tflops"]), "bf16": float(d["bf16_tflops"])},
                "sustained_tflops": {"fp16": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                                     "bf16": float(d.get("bf16_tflops_sustained", d["bf16_tflops"]))},
                "source": "MEASURED_PEAKS.json",
            }
        from .calibrate import cache_file

        cached = cache_file(target_id)
        if cached.is_file():
            return json.loads(cached.read_text())
        return json.loads((ROOT / "targets" / target_id / "calibration.json").read_text())

    def roofline(self, task: Any, time_s: float, calibration: dict) -> dict:
        """Where one measured time sits against the B200's memory and compute lower bounds
        (tcenv/backends/metal/profile.py:251-283 semantics).  ``task`` carries ``min_bytes``,
        ``flops`` and ``dtype`` (attributes or mapping keys)."""
        get = (lambda k, d=None: task.get(k, d)) if isinstance(task, Mapping) else (lambda k, d=None: getattr(task, k, d))
        min_bytes = float(get("min_bytes", 0) or 0)
        flops = float(get("flops", 0) or 0)
        dtype = get("dtype", "fp16")
        # With the task's read/write split, the achievable bandwidth follows its mix
        # (profile.py:233-248); without it, the copy figure.
        rd, wr = get("read_bytes"), get("write_bytes")
        if rd is not None and wr is not None:
            from .calibrate import effective_peak_gbps

            peak_bw = effective_peak_gbps(rd, wr, calibration) * 1e9
        else:
            peak_bw = float(calibration.get("copy_gbs")) * 1e9
        peak_fl = float(calibration["peak_tflops"].get(dtype, calibration["peak_tflops"]["fp16"])) * 1e12
        t_mem = min_bytes / peak_bw if min_bytes else 0.0
        t_cmp = flops / peak_fl if flops else 0.0
        t_lb = max(t_mem, t_cmp)
        return {
            "bound": "compute" if t_cmp > t_mem else "memory",
            "min_bytes": min_bytes,
            "flops": flops,
            "arithmetic_intensity": flops / min_bytes if min_bytes else 0.0,
            "ridge_intensity": peak_fl / peak_bw,
            "achieved_gbps": min_bytes / time_s / 1e9 if time_s > 0 else 0.0,
            "bandwidth_fraction": (min_bytes / time_s) / peak_bw if time_s > 0 else 0.0,
            "achieved_tflops": flops / time_s / 1e12 if time_s > 0 and flops else 0.0,
            "compute_fraction": (flops / time_s) / peak_fl if time_s > 0 and flops else 0.0,
            "lower_bound_us": t_lb * 1e6,
            "time_over_lower_bound": time_s / t_lb if t_lb > 0 else None,
            "peak_gbps_measured": peak_bw / 1e9,
            "peak_tflops_measured": peak_fl / 1e12,
            "bound_kind": "reference_algorithm",
        }

    def describe(self, contract: Any = None) -> str:
        return "CUDA sm_100a backend: candidates are extern \"C\" __global__ kernels taking the ABI tensors in order."

    def abi_stub(self, contract: Any) -> str:
        """An `extern "C"` kernel signature with the contract's tensors in ABI order."""
        ctype = {"fp16": "__half", "bf16": "__nv_bfloat16", "fp32": "float", "i32": "int", "u32": "unsigned int"}
        tensors = contract["tensors"] if isinstance(contract, Mapping) else contract.tensors
        params = []
        for t in tensors:
            name, dtype, access = (t["name"], t["dtype"], t.get("access", "read")) if isinstance(t, Mapping) else (t.name, t.dtype, t.access)
            const = "const " if access == "read" else ""
            params.append(f"{const}{ctype.get(dtype, 'void')}* __restrict__ {name}")
        return 'extern "C" __global__ void candidate(' + ", ".join(params) + ");"

    def compiler_baseline(self, task_name, dtype, size, baseline_us, candidate_us) -> dict:
        return {}

    def assemble(self, contract: Any, source: str) -> tuple[str, int]:
        """The compilation unit: the runtime headers, then the candidate (tcenv/backends/base.py:236)."""
        return self.runtime_headers + source, self.runtime_headers.count("\n")

    def rewrite_compiler_lines(self, contract: Any, message: str, header_lines: int) -> str:
        """Map nvcc's ``file(LINE)`` / ``file:LINE:`` positions back to candidate lines (base.py:245);
        a position inside the header is reported as such."""

        def fix(open_: str, close: str):
            def repl(m: re.Match) -> str:
                line = int(m.group(2)) - header_lines
                return f"{m.group(1)}{open_}{line}{close}" if line >= 1 else f"{m.group(1)}{open_}<runtime header>{close}"
            return repl

        message = re.sub(r"(\S+?\.cu)\((\d+)\)", fix("(", ")"), message)
        return re.sub(r"(\S+?\.cu):(\d+):", fix(":", ":"), message)

    # Validation pass (base.py:98-118).  CUDA builds are not instrumented, so the shared-memory
    # figure a validation build reports is the real one; the only filter is the reference's.
    def is_instrumented_size_only(self, violations: list[str]) -> bool:
        from . import kernel_stats

        return kernel_stats.only_static_smem_limit(violations)

    def validation_problems(self, violations: list[str], static_bytes: list[int], max_tg_memory: int) -> list[str]:
        """Drop the static shared-memory message when every entry's static bytes fit the limit."""
        from . import kernel_stats

        if all(int(b) <= int(max_tg_memory) for b in static_bytes):
            return [v for v in violations if kernel_stats.STATIC_SMEM_LIMIT not in v]
        return list(violations)

    def validation_summary(self, *, size_only: bool, target: Any) -> str:
        if not size_only:
            return "clean"
        limits = target.limits if hasattr(target, "limits") else target["limits"]
        limit = limits.max_threadgroup_memory_bytes if hasattr(limits, "max_threadgroup_memory_bytes") else limits["max_threadgroup_memory_bytes"]
        return f"skipped: only the static shared-memory figure was over the {limit} B limit"

    def coverage(self, task: Any, results: list, source: str, toolchain: dict) -> dict:
        """Sampled cases (the task's generated cases and seeds), not a domain sweep (base.py:207)."""
        return {"kind": "sampling", "scope": ""}

    def artifact_builder(self, *, kernel_contract: Any = None, math: str = "fast", kernel_names: Any = None,
                         diagnostic_profile: str | None = None, specialization: Any = None):
        """The one builder of this backend (base.py:271): the cuda-single nvcc build."""
        from .track_factory import CudaTrackBuilder

        if diagnostic_profile is not None:
            raise ValueError(f"no diagnostic build profile {diagnostic_profile!r} is registered for cuda-sm100")
        if math not in ("fast", "safe"):
            raise ValueError(f"math mode must be fast or safe, got {math!r}")
        return CudaTrackBuilder(extra_flags=("--use_fast_math",) if math == "fast" else ())

    def check_abi(self, contract: Any, kernels: list[Any], *, target: Any = None, device_info: Mapping[str, Any] | None = None,
                  spec: Any = None, validation: bool = False) -> list[str]:
        """Compiled entries (``kernel_stats.KernelResources``) against the launch stages ``spec``
        and the target's limits (base.py:293): every stage's entry compiled, threads, shared memory
        and registers within one SM."""
        from . import kernel_stats

        limits = getattr(target, "limits", None) if target is not None else None
        max_threads = int(getattr(limits, "max_threads_per_threadgroup", kernel_stats.MAX_THREADS_PER_CTA))
        max_smem = int(getattr(limits, "max_threadgroup_memory_bytes", kernel_stats.MAX_SMEM_PER_CTA))
        live = int((device_info or {}).get("max_smem_per_block_optin") or 0)
        if live:
            max_smem = min(max_smem, live)
        by_name = {k.name: k for k in kernels}
        stages = list(spec or [])
        if stages:
            problems = kernel_stats.check_stages(by_name, stages, max_threads=max_threads, max_smem=max_smem)
        else:
            problems = [f"entry `{k.name}`: {kernel_stats.STATIC_SMEM_LIMIT} ({k.static_smem} > {max_smem} bytes)"
                        for k in kernels if k.static_smem > max_smem]
        if validation:
            problems = self.validation_problems(problems, [k.static_smem for k in kernels], max_smem)
        return problems

    def pipeline_stats(self, kernel: Any, contract: Any, device_info: Mapping[str, Any], *, kernel_source: str | None = None) -> dict:
        """One compiled entry under one launch stage ``contract`` (base.py:305)."""
        from . import kernel_stats

        return kernel_stats.stats(kernel, contract, device_info)

    def pipeline_stats_many(self, pairs: list, device_info: Mapping[str, Any], *, kernel_source: str | None = None) -> dict:
        from . import kernel_stats

        return kernel_stats.stats_many(pairs, device_info)

    # ---- child-process hooks (device) ----------------------------------------------------------

    def set_heartbeat_hooks(self, *, on_compile=None, on_launch=None) -> None:
        """Install ``(begin, end)`` pairs run around every nvcc build and every synchronised launch
        (a correctness case, a k-launch timing batch); an omitted pair is left as it is
        (tcenv/backends/base.py:194 contract)."""
        from . import heartbeat

        if on_compile is not None:
            heartbeat.set_compile_hooks(*on_compile)
        if on_launch is not None:
            heartbeat.set_launch_hooks(*on_launch)

    def context(self):
        import torch

        from . import _native

        _native.load()
        return torch.device("cuda", torch.cuda.current_device())

    def compile_error(self):
        return CudaCompileError

    def runtime_error(self):
        return CudaRuntimeError

    def probe(self, ctx: Any = None, target: Any = None) -> DeviceInfo:
        from . import _native

        device = getattr(ctx, "index", None) or 0
        info = _native.device_info(int(device))
        matches = self.device_matches(target or {"match_name_contains": "B200"}, info)
        limits = {
            "max_threads_per_threadgroup": info["max_threads_per_block"],
            "max_threadgroup_memory_bytes": info["max_smem_per_block_optin"],
            "sm_count": info["sm_count"],
            "l2_bytes": info["l2_bytes"],
        }
        return DeviceInfo(backend=self.id, name=info["name"], family=f"sm_{info['cc_major']}{info['cc_minor']}", limits=limits,
                          raw=info, matches=matches, match_error="" if matches else f"{info['name']} is not a B200")

    def rotation_sets(self, task: Any) -> int:
        """Enough argument sets that one rotation exceeds twice the 126 MB L2 (≤ 16 sets)."""
        get = (lambda k, d=None: task.get(k, d)) if isinstance(task, Mapping) else (lambda k, d=None: getattr(task, k, d))
        per = float(get("min_bytes", 0) or 1)
        return int(max(1, min(16, -(-2 * 126 * 2**20 // per))))

    def run_correctness(self, ctx: Any, launch: Callable[[list[int]], None], specs, cases, *, rtol: float, atol_rel: float,
                        exact: bool = False, output_dtypes: Mapping[str, str] | None = None) -> list:
        """Run every case (``(name, inputs, refs, scales)``) through the three guarded trials."""
        from .runtime import CorrectnessRunner

        from .heartbeat import launching

        runner = CorrectnessRunner(specs, launch, ctx, output_dtypes=output_dtypes)
        results = []
        for name, inputs, refs, scales in cases:
            with launching():
                results.append(runner.run_case(name, inputs, refs, scales, rtol, atol_rel, exact))
            if not results[-1].ok:
                break  # the reference stops at the first failing case
        return results

    def prepare_bench(self, desc, pointer_sets, *, use_graph: bool = False) -> Callable[[int], float]:
        """The candidate runner for the timing protocol: k launches over rotating argument sets
        timed between CUDA events by ``sf_run_batch`` (the taic_metal_run_batch replacement)."""
        import torch

        from . import _native

        stream = torch.cuda.current_stream().cuda_stream

        from .heartbeat import launching

        def run_k(k: int) -> float:
            with launching():
                return _native.run_batch(desc, pointer_sets, k, stream, use_graph=use_graph)

        return run_k
