"""Shape portfolios of CUDA candidates: pack a source tree, check its coverage, dispatch, account.

The layout and the rules follow the reference's portfolio assembly
(tcenv/portfolio_assembly/assembly.py:132-345, ``_load_coverage`` / ``_fallback_shape`` /
``_portfolio_document`` below it) with cuda-single sources in place of Metal ones::

    <src>/coverage.json            {"schema_id": "tcenv.portfolio-assembly.coverage.1",
                                    "planner": {"id": ..., "version": n},
                                    "variants": [{"variant_key": k, "guard": <predicate term>,
                                                  "bucket_key": b (optional)}, ...],
                                    "fallback": {"kind": "refuse", "reasons": [...]} or
                                                {"kind": "registered_implementation", "reasons": [...],
                                                 "implementation_id": ..., "implementation_version": n}}
    <src>/variants/<k>/kernel.cu   one single-source candidate per variant
    <src>/fallback/kernel.cu       the registered implementation's source (``fallbacks.render``)

Guards are predicate terms of ``expr`` over the task's symbols.  A portfolio kernel takes the
task's ABI tensors in opspec order followed by the symbols as ``long long`` in ``spec_params``
order, and its ``taic-launch`` values may be expressions over the symbols, so one build serves
every shape its guard admits.

* ``pack`` validates the tree (closed key sets, variant-key pattern, at most 16 variants, unique
  keys, one guard per bucket, registered fallback reasons, every source through the cuda-single
  builder's pre-compile checks) and returns the parent: entries plus the ``portfolio.json``
  document (guard digests, the domain-plan digest of the sizes it was packed for).
* ``check`` evaluates every guard on every point of the domain (size x usage of the task's
  opspec): each point must go to exactly one variant, or to an implementation fallback when no
  guard matches; overlaps, guard errors, variants that match no point and unresolvable launches
  are problems.
* ``to_portfolio`` gives the exact-dispatch ``portfolio.Portfolio`` of a parent (overlap and
  guard errors are dispatch failures, no ranking), and ``measure`` runs and times every benchmark
  point on the GPU against the task's torch baseline, so ``PerformanceReport``'s
  ``effective_end_to_end`` account includes the real time of the shards the fallback serves.
"""

from __future__ import annotations

import base64
import hashlib
import json
import re
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, Mapping, Sequence

from . import expr, fallbacks
from .portfolio import Fallback, Portfolio, Variant

COVERAGE_SCHEMA_ID = "tcenv.portfolio-assembly.coverage.1"
PORTFOLIO_SCHEMA_ID = "cuda-sm100.candidate-portfolio.1"
PORTFOLIO_ENTRY_PATH = "coverage_plan/portfolio.json"
FALLBACK_REASONS = frozenset({"outside_candidate_coverage", "resource_unavailable", "variant_unavailable"})
MAX_VARIANTS = 16
SOURCE_NAME = "kernel.cu"
_VARIANT_KEY = re.compile(r"[a-z0-9][a-z0-9_-]{0,31}")
_COVERAGE_KEYS = frozenset({"schema_id", "planner", "variants", "fallback"})
_VARIANT_ITEM_KEYS = frozenset({"variant_key", "guard", "bucket_key"})
_REFUSE_KEYS = frozenset({"kind", "reasons"})
_IMPLEMENTATION_KEYS = frozenset({"kind", "reasons", "implementation_id", "implementation_version"})


class PortfolioError(ValueError):
    """The source tree, its coverage.json or a parent document breaks the packing contract."""


# ---- the finite domain ------------------------------------------------------------------------


@dataclass(frozen=True)
class Point:
    instance_key: str  # "<dtype>/<size>/<usage>"
    size: str
    usage: str
    names: Mapping[str, int]


def load_opspec(task_dir: str | Path) -> dict[str, Any]:
    return json.loads((Path(task_dir) / "opspec.json").read_text(encoding="utf-8"))


def symbol_order(opspec: Mapping[str, Any]) -> tuple[str, ...]:
    """The kernel-argument order of the symbols: ``spec_params``, else the declared symbols."""
    return tuple(opspec.get("spec_params") or opspec.get("symbols", {}).keys())


def domain(opspec: Mapping[str, Any], dtype: str, sizes: Sequence[str] | None = None) -> tuple[Point, ...]:
    """Every (size, usage) point of the task for ``dtype``, in opspec order."""
    declared = opspec.get("sizes", {})
    chosen = list(sizes) if sizes is not None else list(declared)
    if not chosen or len(set(chosen)) != len(chosen):
        raise PortfolioError(f"sizes must be non-empty and distinct, got {chosen}")
    points = []
    for size in chosen:
        if size not in declared:
            raise PortfolioError(f"size {size!r} is not declared by the task (declared: {sorted(declared)})")
        entry = declared[size]
        names = {k: int(v) for k, v in entry.items() if k != "usage" and isinstance(v, int) and not isinstance(v, bool)}
        # Varlen sizes declare their batch, not its symbols: total_tokens / num_seqs (and NSP1 =
        # num_seqs + 1, the cu_seqlens length) come from seq_lens, or from the capacity of an L2 tier.
        if isinstance(entry.get("capacity"), Mapping):
            names.update(total_tokens=int(entry["capacity"]["total_tokens"]), num_seqs=int(entry["capacity"]["num_seqs"]))
        elif isinstance(entry.get("seq_lens"), list):
            names.update(total_tokens=sum(int(x) for x in entry["seq_lens"]), num_seqs=len(entry["seq_lens"]))
        if "num_seqs" in names:
            names["NSP1"] = names["num_seqs"] + 1
        for usage in entry.get("usage", ["benchmark"]):
            points.append(Point(f"{dtype}/{size}/{usage}", size, usage, names))
    return tuple(points)


def domain_digest(points: Sequence[Point]) -> str:
    doc = [{"instance_key": p.instance_key, "names": dict(sorted(p.names.items()))} for p in points]
    return hashlib.sha256(json.dumps(doc, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


# ---- the parent -------------------------------------------------------------------------------


@dataclass(frozen=True)
class Entry:
    path: str
    role: str
    media_type: str
    data: bytes


@dataclass(frozen=True)
class Parent:
    entries: tuple[Entry, ...]
    document: Mapping[str, Any]

    def entry(self, path: str) -> Entry:
        for e in self.entries:
            if e.path == path:
                return e
        raise PortfolioError(f"the parent has no entry {path!r}")

    def source(self, path: str) -> str:
        return self.entry(path).data.decode("utf-8")

    def to_json(self) -> str:
        return json.dumps({
            "transport": "shape-portfolio",
            "entries": [{"path": e.path, "role": e.role, "media_type": e.media_type,
                         "data": base64.b64encode(e.data).decode("ascii")} for e in self.entries],
        }, sort_keys=True, indent=1)

    @property
    def sha256(self) -> str:
        return hashlib.sha256(self.to_json().encode()).hexdigest()

    @classmethod
    def from_json(cls, text: str) -> "Parent":
        doc = json.loads(text)
        if doc.get("transport") != "shape-portfolio":
            raise PortfolioError("not a shape-portfolio parent")
        entries = tuple(Entry(e["path"], e["role"], e["media_type"], base64.b64decode(e["data"])) for e in doc["entries"])
        manifest = [e for e in entries if e.path == PORTFOLIO_ENTRY_PATH]
        if len(manifest) != 1:
            raise PortfolioError(f"a parent needs exactly one {PORTFOLIO_ENTRY_PATH}")
        return cls(entries, json.loads(manifest[0].data))


def _read_source(path: Path) -> bytes:
    if not path.is_file() or path.is_symlink():
        raise PortfolioError(f"{path}: expected a regular file")
    data = path.read_bytes()
    try:
        data.decode("utf-8")
    except UnicodeDecodeError as exc:
        raise PortfolioError(f"{path}: not UTF-8") from exc
    if not data.strip():
        raise PortfolioError(f"{path}: empty source")
    return data


def _single_source(directory: Path, where: str) -> bytes:
    """A variant (or fallback) directory holds exactly one ``kernel.cu``."""
    if not directory.is_dir() or directory.is_symlink():
        raise PortfolioError(f"{directory}: expected a directory")
    files = sorted(p.relative_to(directory).as_posix() for p in directory.rglob("*") if p.is_file() or p.is_symlink())
    if files != [SOURCE_NAME]:
        raise PortfolioError(f"{directory}: a cuda-single {where} is exactly {SOURCE_NAME}, found {files}")
    data = _read_source(directory / SOURCE_NAME)
    from .track_factory import CudaTrackBuilder, TrackRefused

    try:
        CudaTrackBuilder().check(data.decode("utf-8"))
    except TrackRefused as exc:
        raise PortfolioError(f"{directory / SOURCE_NAME}: {exc}") from exc
    return data


def _load_coverage(path: Path) -> dict[str, Any]:
    try:
        doc = json.loads(_read_source(path))
    except json.JSONDecodeError as exc:
        raise PortfolioError(f"{path}: not JSON: {exc}") from exc
    if not isinstance(doc, dict) or set(doc) != _COVERAGE_KEYS:
        raise PortfolioError(f"{path}: keys must be exactly {sorted(_COVERAGE_KEYS)}")
    if doc["schema_id"] != COVERAGE_SCHEMA_ID:
        raise PortfolioError(f"{path}: schema_id must be {COVERAGE_SCHEMA_ID!r}")
    planner = doc["planner"]
    if (not isinstance(planner, dict) or set(planner) != {"id", "version"} or not isinstance(planner["id"], str)
            or not planner["id"].strip() or isinstance(planner["version"], bool) or not isinstance(planner["version"], int)
            or planner["version"] < 1):
        raise PortfolioError(f"{path}: planner must be {{id: non-empty string, version: positive integer}}")
    variants = doc["variants"]
    if not isinstance(variants, list) or not variants or len(variants) > MAX_VARIANTS:
        raise PortfolioError(f"{path}: variants must be a list of 1..{MAX_VARIANTS} items")
    return doc


def _fallback(doc: Any, root: Path, path: Path) -> tuple[dict[str, Any], bytes | None]:
    if not isinstance(doc, dict) or "kind" not in doc:
        raise PortfolioError(f"{path}: fallback must be an object with a kind")
    reasons = doc.get("reasons")
    if (not isinstance(reasons, list) or not reasons or len(set(reasons)) != len(reasons)
            or any(r not in FALLBACK_REASONS for r in reasons)):
        raise PortfolioError(f"{path}: fallback reasons must be a non-empty list drawn from {sorted(FALLBACK_REASONS)}")
    directory = root / "fallback"
    if doc["kind"] == "refuse":
        if set(doc) != _REFUSE_KEYS:
            raise PortfolioError(f"{path}: a refuse fallback has only kind and reasons")
        if directory.exists():
            raise PortfolioError(f"{directory}: a refuse fallback has no fallback directory")
        return {"kind": "refuse", "implementation_id": None, "implementation_version": None, "entries": [],
                "reasons": list(reasons)}, None
    if doc["kind"] != "registered_implementation":
        raise PortfolioError(f"{path}: unknown fallback kind {doc['kind']!r}")
    if set(doc) != _IMPLEMENTATION_KEYS:
        raise PortfolioError(f"{path}: a registered_implementation fallback has exactly {sorted(_IMPLEMENTATION_KEYS)}")
    impl, version = doc["implementation_id"], doc["implementation_version"]
    if not isinstance(impl, str) or not impl.strip() or isinstance(version, bool) or not isinstance(version, int) or version < 1:
        raise PortfolioError(f"{path}: implementation_id must be a non-empty string and implementation_version >= 1")
    data = _single_source(directory, "fallback")
    return {"kind": "registered_implementation", "implementation_id": impl, "implementation_version": version,
            "entries": [f"fallback/{SOURCE_NAME}"], "reasons": list(reasons)}, data


def pack(src: str | Path, points: Sequence[Point]) -> Parent:
    """Validate ``src`` and build the parent (sources + ``coverage_plan/portfolio.json``)."""
    root = Path(src)
    cov_path = root / "coverage.json"
    coverage = _load_coverage(cov_path)
    vdir = root / "variants"
    if not vdir.is_dir():
        raise PortfolioError(f"{vdir}: expected a variants directory")
    on_disk = sorted(p.name for p in vdir.iterdir() if not p.name.startswith("."))
    declared: dict[str, dict[str, Any]] = {}
    for i, item in enumerate(coverage["variants"]):
        where = f"{cov_path}: variants[{i}]"
        if not isinstance(item, dict) or not set(item) <= _VARIANT_ITEM_KEYS or "variant_key" not in item or "guard" not in item:
            raise PortfolioError(f"{where}: allows only variant_key, guard and an optional bucket_key")
        key = item["variant_key"]
        if not isinstance(key, str) or not _VARIANT_KEY.fullmatch(key):
            raise PortfolioError(f"{where}: variant_key {key!r} must match [a-z0-9][a-z0-9_-]{{0,31}}")
        if key in declared:
            raise PortfolioError(f"{cov_path}: variant_key {key!r} is repeated")
        declared[key] = item
    if sorted(declared) != on_disk:
        raise PortfolioError(f"{cov_path}: variant keys {sorted(declared)} do not match the directories {on_disk}")
    entries: list[Entry] = []
    variants_doc = []
    buckets: dict[str, str] = {}
    for key, item in declared.items():
        try:
            expr.guard(item["guard"], where=f"guard of {key}")
            gdig = expr.digest(item["guard"])
        except expr.ExprError as exc:
            raise PortfolioError(f"{cov_path}: {exc}") from exc
        bucket = item.get("bucket_key", key)
        if not isinstance(bucket, str) or not bucket.strip() or len(bucket) > 128:
            raise PortfolioError(f"{cov_path}: bucket_key of {key} must be a non-empty string of at most 128 characters")
        if buckets.setdefault(bucket, gdig) != gdig:
            raise PortfolioError(f"{cov_path}: bucket {bucket!r} is used with two different guards")
        data = _single_source(vdir / key, f"variant {key}")
        path = f"variants/{key}/{SOURCE_NAME}"
        entries.append(Entry(path, "device_kernel", "text/x-cuda", data))
        variants_doc.append({"variant_key": key, "bucket_key": bucket, "guard": {"expr": item["guard"], "digest": gdig},
                             "entries": [path]})
    fb_doc, fb_data = _fallback(coverage["fallback"], root, cov_path)
    if fb_data is not None:
        entries.append(Entry(f"fallback/{SOURCE_NAME}", "device_kernel", "text/x-cuda", fb_data))
    document = {
        "schema_id": PORTFOLIO_SCHEMA_ID,
        "domain_plan_digest": domain_digest(points),
        "domain": [p.instance_key for p in points],
        "planner": dict(coverage["planner"]),
        "coverage_plan": {"buckets": [{"bucket_key": b, "guard_digest": d} for b, d in buckets.items()]},
        "variants": variants_doc,
        "fallback": fb_doc,
    }
    entries.sort(key=lambda e: e.path)
    entries.append(Entry(PORTFOLIO_ENTRY_PATH, "launch", "application/json",
                         json.dumps(document, indent=2, sort_keys=True).encode() + b"\n"))
    return Parent(tuple(entries), document)


def write_fallback(src: str | Path, task: str, dtype: str, attrs: Mapping[str, float] | None = None) -> dict[str, Any]:
    """Materialise the registered fallback of ``task`` as ``<src>/fallback/kernel.cu`` and return the
    coverage.json ``fallback`` stanza that names it."""
    directory = Path(src) / "fallback"
    directory.mkdir(parents=True, exist_ok=True)
    (directory / SOURCE_NAME).write_text(fallbacks.render(task, dtype, attrs), encoding="utf-8")
    return {"kind": "registered_implementation", "reasons": ["outside_candidate_coverage"],
            "implementation_id": fallbacks.implementation_id(task), "implementation_version": fallbacks.VERSION}


# ---- dispatch and coverage check --------------------------------------------------------------


def to_portfolio(parent: Parent) -> Portfolio:
    """Exact dispatch over the parent's guards (``portfolio.Portfolio``): variant ``name`` is the
    variant_key, the fallback's name its implementation id."""
    variants = []
    for v in parent.document["variants"]:
        node = expr.guard(v["guard"]["expr"], where=f"guard of {v['variant_key']}")
        variants.append(Variant(v["variant_key"], (lambda n, node=node: expr.evaluate(node, n))))
    fb = parent.document["fallback"]
    fallback = None
    if fb["kind"] == "registered_implementation":
        fallback = Fallback(fb["implementation_id"], handles=tuple(fb["reasons"]))
    return Portfolio(tuple(variants), fallback)


def selected_source(parent: Parent, record: Any) -> str:
    """The source a dispatch record selects."""
    if record.provider == "candidate":
        return parent.source(f"variants/{record.selected}/{SOURCE_NAME}")
    if record.provider == "fallback":
        return parent.source(f"fallback/{SOURCE_NAME}")
    raise PortfolioError(f"dispatch selected nothing: {record.outcome} ({record.detail})")


@dataclass(frozen=True)
class CheckRow:
    instance_key: str
    size: str
    usage: str
    provider: str  # candidate | fallback | none
    variant_key: str | None


@dataclass(frozen=True)
class CheckReport:
    ok: bool
    problems: tuple[str, ...]
    rows: tuple[CheckRow, ...]
    domain_plan_digest: str

    def document(self) -> dict[str, Any]:
        return {"ok": self.ok, "problems": list(self.problems), "domain_plan_digest": self.domain_plan_digest,
                "rows": [r.__dict__ for r in self.rows]}


def check(parent: Parent, points: Sequence[Point]) -> CheckReport:
    """Coverage of ``points`` by the parent's guards and the projection of every used source's
    launch block onto the points it serves (CPU only; never raises on a failed check)."""
    from .backend import CudaBackend, parse_launch_templates

    digest = domain_digest(points)
    problems: list[str] = []
    if parent.document.get("domain_plan_digest") != digest:
        problems.append("the parent was packed for another domain (pack and check need the same sizes)")
    port = to_portfolio(parent)
    rows: list[CheckRow] = []
    hit: set[str] = set()
    backend = CudaBackend()
    for p in points:
        rec = port.resolve(p.names)
        if rec.outcome in ("candidate", "fallback"):
            if rec.provider == "candidate":
                hit.add(rec.selected)
            try:
                stages = [t.resolve(p.names) for t in parse_launch_templates(selected_source(parent, rec))]
                problems.extend(f"{p.instance_key}: {msg}" for msg in backend.validate_launch(stages, {}))
            except (ValueError, expr.ExprError) as exc:
                problems.append(f"{p.instance_key}: launch of {rec.selected} does not resolve: {exc}")
            rows.append(CheckRow(p.instance_key, p.size, p.usage, rec.provider, rec.selected if rec.provider == "candidate" else None))
            continue
        if rec.outcome == "dispatch_overlap":
            problems.append(f"{p.instance_key}: more than one variant matches ({rec.detail})")
        elif rec.outcome == "dispatch_unknown":
            problems.append(f"{p.instance_key}: a guard cannot be evaluated ({rec.detail})")
        else:
            problems.append(f"{p.instance_key}: no variant matches and there is no implementation fallback")
        rows.append(CheckRow(p.instance_key, p.size, p.usage, "none", None))
    for v in parent.document["variants"]:
        if v["variant_key"] not in hit:
            problems.append(f"{v['variant_key']}: matches no point of the domain")
    return CheckReport(not problems, tuple(problems), tuple(rows), digest)


# ---- measurement (GPU) --------------------------------------------------------------------------


@dataclass
class ShardRun:
    point: Point
    provider: str
    selected: str
    candidate_us: float
    baseline_us: float
    correct: bool
    detail: str = ""
    timing_uncertain: bool = False
    candidate_cv: float = 0.0
    baseline_cv: float = 0.0
    attempts: int = 0
    source_sha256: str = ""
    cache_hit: bool = False


def storage_dtype(name: str, task_dtype: str):
    """The torch dtype holding an opspec tensor dtype (``T`` is the instance's dtype; ``u32`` is held
    as int32, the same 4 bytes)."""
    import torch

    table = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32, "i32": torch.int32, "u32": torch.int32}
    key = task_dtype if name == "T" else name
    if key not in table:
        raise PortfolioError(f"no storage dtype for {name!r}")
    return table[key]


def output_specs(opspec: Mapping[str, Any], point: Point) -> dict[str, tuple[tuple[int, ...], Any]]:
    """Shape (dims evaluated on the point's symbols) and torch dtype of every output, in ABI order."""
    dtype = point.instance_key.split("/")[0]
    out = {}
    for name, t in opspec["tensors"].items():
        if t["role"] == "output":
            out[name] = (tuple(int(expr.evaluate_term(d, point.names)) for d in t["dims"]), storage_dtype(t["dtype"], dtype))
    return out


def _timed(candidate: Callable[[], Any], baseline: Callable[[], Any], reps: int):
    """Per-launch device microseconds of candidate and baseline through the harness timing
    protocol (``protocol.measure_interleaved``: batches sized to ~15 ms, interleaved repetitions,
    up to three attempts).  Returns (candidate stats, baseline stats, noisy, attempts); noisy is
    True when the kept attempt's CV is above 5 %."""
    from . import protocol
    from .gpulock import gpu_lock
    from .heartbeat import launching

    def batch(fn: Callable[[], Any]) -> Callable[[int], float]:
        run_k = protocol.cuda_event_runner(lambda i: fn())

        def bracketed(k: int) -> float:
            with launching():  # one synchronised k-launch batch
                return run_k(k)

        return bracketed

    runners = {"candidate": batch(candidate), "baseline": batch(baseline)}
    with gpu_lock("portfolio shard timing"):  # exclusive on this GPU for the whole measurement
        noise, stats, attempts = protocol.measure_interleaved(runners, reps=reps)
    return stats["candidate"], stats["baseline"], noise > protocol.NOISY_CV, attempts


def run_point(parent: Parent, opspec: Mapping[str, Any], point: Point, inputs: Mapping[str, Any], *,
              baseline: Callable[..., Any] | None,
              verify: Callable[[Point, Mapping[str, Any], Mapping[str, Any]], tuple[bool, str]],
              reps: int = 15, use_cache: bool = True, builds: dict[str, Any] | None = None) -> ShardRun:
    """Dispatch ``point``, build the selected source (``use_cache=False``: a fresh nvcc build), run
    it once on ``inputs`` (CUDA tensors by ABI name; outputs are allocated from the opspec), verify,
    and — with a ``baseline`` — time candidate and baseline through the interleaved protocol."""
    import ctypes

    import torch

    from .candidates import Module
    from .track_factory import CudaTrackBuilder

    rec = to_portfolio(parent).resolve(point.names)
    source = selected_source(parent, rec)
    key = hashlib.sha256(source.encode()).hexdigest()
    builds = {} if builds is None else builds
    if key not in builds or not use_cache:
        builds[key] = CudaTrackBuilder().build(source, use_cache=use_cache)
    build = builds[key]
    outputs = {name: torch.empty(shape, dtype=dt, device="cuda") for name, (shape, dt) in output_specs(opspec, point).items()}
    ptrs = [(inputs[n] if n in inputs else outputs[n]).data_ptr() for n in opspec["tensors"]]
    stream = torch.cuda.current_stream().cuda_stream
    module = Module(build.image)
    scalars = [ctypes.c_longlong(point.names[s]) for s in symbol_order(opspec)]
    bound = [module.bind(st.kernel, st.grid, st.threads, ptrs + scalars, smem=st.smem, stream=stream)
             for st in (t.resolve(point.names) for t in build.stages)]

    def run() -> None:
        for b in bound:
            b()

    from .heartbeat import launching

    with launching():  # an evaluation worker's launch deadline covers the verified run
        run()
        torch.cuda.synchronize()
    ok, detail = verify(point, inputs, outputs)
    shard = ShardRun(point, rec.provider, rec.selected, 0.0, 0.0, ok, detail, source_sha256=key, cache_hit=build.cache_hit)
    if baseline is not None:
        ins = [inputs[n] for n, t in opspec["tensors"].items() if t["role"] == "input"]
        cand, base, noisy, attempts = _timed(run, lambda: baseline(*ins), reps)
        shard.candidate_us, shard.baseline_us = cand.median_s * 1e6, base.median_s * 1e6
        shard.candidate_cv, shard.baseline_cv = cand.cv, base.cv
        shard.timing_uncertain, shard.attempts = noisy, attempts
    return shard


def measure(parent: Parent, opspec: Mapping[str, Any], points: Sequence[Point], *,
            make_inputs: Callable[[Point], Mapping[str, Any]],
            baseline: Callable[..., Any],
            verify: Callable[[Point, Mapping[str, Any], Mapping[str, Any]], tuple[bool, str]],
            reps: int = 15) -> list[ShardRun]:
    """``run_point`` over every benchmark point of ``points`` (one build per distinct source).

    ``make_inputs(point)`` gives the input tensors (CUDA, by ABI name); ``baseline(*inputs in ABI
    order)`` is the task's timing baseline; ``verify(point, inputs, outputs)`` returns ``(ok, detail)``."""
    builds: dict[str, Any] = {}
    return [run_point(parent, opspec, p, make_inputs(p), baseline=baseline, verify=verify, reps=reps, builds=builds)
            for p in points if p.usage == "benchmark"]


def performance(runs: Sequence[ShardRun]):
    """The reference's two accounts over the measured shards (``portfolio.PerformanceReport``)."""
    from .portfolio import PerformanceReport, ShardMeasurement

    return PerformanceReport.evaluate([
        ShardMeasurement(r.point.instance_key, r.point.usage, r.provider, r.candidate_us, r.baseline_us,
                         timing_uncertain=r.timing_uncertain, correctness_ok=r.correct)
        for r in runs
    ])


# ---- command line ---------------------------------------------------------------------------------


def main(argv: Sequence[str] | None = None) -> int:
    """``python -m shapeforge_b200.portfolio_pack pack|check`` (the reference's ``portfolio-pack`` /
    ``portfolio-check`` commands for CUDA sources).

    ``pack SRC --task-dir T --dtype D [--sizes a,b] --out PARENT.json`` validates the tree and writes
    the parent; ``check PARENT.json --task-dir T --dtype D [--sizes a,b]`` prints the coverage report
    as JSON and exits 1 when it has problems."""
    import argparse
    import sys

    ap = argparse.ArgumentParser(prog="python -m shapeforge_b200.portfolio_pack")
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name in ("pack", "check"):
        p = sub.add_parser(name)
        p.add_argument("path", help="source tree (pack) or parent JSON (check)")
        p.add_argument("--task-dir", required=True, help="directory holding the task's opspec.json")
        p.add_argument("--dtype", required=True, choices=("fp16", "bf16"))
        p.add_argument("--sizes", default=None, help="comma-separated sizes (default: every declared size)")
        if name == "pack":
            p.add_argument("--out", required=True)
    args = ap.parse_args(argv)
    points = domain(load_opspec(args.task_dir), args.dtype, args.sizes.split(",") if args.sizes else None)
    try:
        if args.cmd == "pack":
            parent = pack(args.path, points)
            Path(args.out).write_text(parent.to_json() + "\n", encoding="utf-8")
            print(json.dumps({"parent_sha256": parent.sha256, "domain_plan_digest": parent.document["domain_plan_digest"],
                              "variants": [v["variant_key"] for v in parent.document["variants"]]}))
            return 0
        parent = Parent.from_json(Path(args.path).read_text(encoding="utf-8"))
        report = check(parent, points)
        print(json.dumps(report.document(), indent=1))
        return 0 if report.ok else 1
    except PortfolioError as exc:
        print(f"portfolio: {exc}", file=sys.stderr)
        return 2


if __name__ == "__main__":
    raise SystemExit(main())
