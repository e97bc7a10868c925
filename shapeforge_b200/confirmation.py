"""Fresh confirmation of a portfolio's shards, and publication into a ``kernels/b200`` catalog.

A shard's search result (the candidate evaluated on the search seed's inputs) counts only after an
independent confirmation: the same source rebuilt without the cubin cache, run on inputs from a
fresh seed, verified again and timed again.  The verdict rules restate the subject confirmation
of taic/portfolio_confirmation.py:66-116 (``_subject_verdict``):

* both evaluations ``ok`` and neither served from a cache; native full builds of the same
  candidate source (sha256);
* both on the subject's dtype / size / mode (``full`` for a benchmark instance, ``quick`` for a
  golden one) and target;
* the search evaluation on ``SEARCH_SEED`` (7), the confirmation on a different, fresh seed;
* for a benchmark instance, the confirmation's timing must not be uncertain (kept attempt CV <= 5 %)
  and it took 1..3 attempts;
* a fallback shard never credits a variant, a candidate shard always does.

The fresh seed is an HMAC of the domain-plan digest and the instance key under the run's master
seed (the reference derives unseen-instance seeds from a master seed the same way, and never
writes the master seed into a document).  Each subject document carries a digest over its
content, so a published document that was edited afterwards fails ``verify_subject``.

``publish`` writes, only when every benchmark subject is confirmed and the performance report is
publishable::

    <catalog>/b200/<task>/<dtype>/<parent sha256[:16]>/
        parent.json        the packed portfolio (transport form)
        performance.json   the accounts and the per-shard times
        subjects/<size>-<usage>.json
        manifest.json      task, dtype, target, parent sha256, domain-plan digest, subject digests
"""

from __future__ import annotations

import hashlib
import hmac
import json
from pathlib import Path
from typing import Any, Callable, Mapping, Sequence

from . import portfolio_pack as pp

SEARCH_SEED = 7
BENCH_ATTEMPTS = 3
QUIET_CV = 0.05
TARGET_ID = "b200"
SUBJECT_SCHEMA_ID = "cuda-sm100.portfolio.subject-confirmation.1"
MAX_SAFE_INTEGER = (1 << 53) - 1


def _canonical(doc: Any) -> bytes:
    return json.dumps(doc, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()


def fingerprint(doc: Any) -> str:
    return hashlib.sha256(_canonical(doc)).hexdigest()


def fresh_seed(master_seed: int, domain_plan_digest: str, instance_key: str) -> int:
    """The confirmation seed of one instance: HMAC-SHA256 keyed by the master seed over the plan
    digest and the instance key, 53 bits, never equal to the search seed."""
    msg = _canonical({"purpose": "fresh-confirmation-seed", "domain_plan_digest": domain_plan_digest,
                      "instance_key": instance_key})
    key = int(master_seed).to_bytes(16, "big", signed=True)
    seed = int.from_bytes(hmac.new(key, msg, hashlib.sha256).digest()[:8], "big") & MAX_SAFE_INTEGER
    return seed + 1 if seed == SEARCH_SEED else seed


def report(run: "pp.ShardRun", *, seed: int, target_id: str = TARGET_ID) -> dict[str, Any]:
    """An evaluation report of one shard run (the fields the verdict reads)."""
    p = run.point
    dtype, size, usage = p.instance_key.split("/")
    doc = {
        "status": "ok" if run.correct else "incorrect",
        "detail": run.detail,
        "cache_hit": bool(run.cache_hit),
        "build": {"shape": "full", "build_kind": "native", "candidate_sha256": run.source_sha256},
        "dtype": dtype, "size": size, "mode": "full" if usage == "benchmark" else "quick",
        "target_id": target_id, "seed": int(seed), "provider": run.provider, "selected": run.selected,
    }
    if usage == "benchmark":
        doc["benchmark"] = {
            "noisy": bool(run.timing_uncertain), "attempts": int(run.attempts),
            "candidate": {"median_us": run.candidate_us, "cv": run.candidate_cv},
            "baseline": {"median_us": run.baseline_us, "cv": run.baseline_cv},
        }
    return doc


def timing_is_uncertain(rep: Mapping[str, Any]) -> bool:
    bench = rep.get("benchmark")
    if not bench or bench.get("noisy") is True:
        return True
    cand = bench.get("candidate") or {}
    return not isinstance(cand.get("cv"), (int, float)) or cand["cv"] > QUIET_CV


def subject_verdict(doc: Mapping[str, Any]) -> tuple[str, str | None]:
    """``("confirmed", None)`` or ``("rejected", reason)`` from the two raw reports."""
    search, conf = doc["search_report"], doc["confirmation_report"]
    parts = doc["instance_key"].split("/")
    if len(parts) != 3 or doc["usage"] != parts[2]:
        return "rejected", "instance_key_mismatch"
    mode = "full" if doc["usage"] == "benchmark" else "quick"
    for period, rep in (("search", search), ("confirmation", conf)):
        if rep.get("status") != "ok":
            return "rejected", f"{period}_status_not_ok"
        if rep.get("cache_hit") is not False:
            return "rejected", "cache_hit"
        build = rep.get("build") or {}
        if build.get("shape") != "full" or build.get("build_kind") != "native":
            return "rejected", "confirmation_ineligible"
        if build.get("candidate_sha256") != doc["candidate_sha256"]:
            return "rejected", "candidate_sha256_mismatch"
        if rep.get("dtype") != parts[0] or rep.get("size") != parts[1]:
            return "rejected", "instance_key_mismatch"
        if rep.get("mode") != mode:
            return "rejected", "measurement_mode_mismatch"
        if rep.get("target_id") != doc["target_id"]:
            return "rejected", "target_mismatch"
        if rep.get("provider") != doc["provider"]:
            return "rejected", "provider_mismatch"
    if doc["search_seed"] != SEARCH_SEED or search.get("seed") != SEARCH_SEED or conf.get("seed") != doc["confirmation_seed"]:
        return "rejected", "seed_mismatch"
    if doc["search_seed"] == doc["confirmation_seed"]:
        return "rejected", "not_fresh"
    if doc["usage"] == "benchmark":
        if timing_is_uncertain(conf):
            return "rejected", "timing_uncertain"
        attempts = (conf.get("benchmark") or {}).get("attempts")
        if type(attempts) is not int or not 1 <= attempts <= BENCH_ATTEMPTS:
            return "rejected", "invalid_attempt_count"
    if doc["provider"] == "fallback" and doc["credits_variant"] is not False:
        return "rejected", "fallback_credits_variant"
    if doc["provider"] == "candidate" and doc["credits_variant"] is not True:
        return "rejected", "variant_credit_mismatch"
    return "confirmed", None


def _finalize(doc: dict[str, Any]) -> dict[str, Any]:
    out = {k: v for k, v in doc.items() if k not in ("status", "reason", "confirmation_digest")}
    out["status"], out["reason"] = subject_verdict(out)
    out["confirmation_digest"] = fingerprint(out)
    return out


def subject(search_run: "pp.ShardRun", confirmation_run: "pp.ShardRun", *, confirmation_seed: int,
            target_id: str = TARGET_ID) -> dict[str, Any]:
    """The subject document of one instance from its search and confirmation runs."""
    p = search_run.point
    return _finalize({
        "schema_id": SUBJECT_SCHEMA_ID,
        "instance_key": p.instance_key,
        "usage": p.usage,
        "provider": search_run.provider,
        "selected": search_run.selected,
        "candidate_sha256": search_run.source_sha256,
        "credits_variant": search_run.provider == "candidate",
        "target_id": target_id,
        "search_seed": SEARCH_SEED,
        "confirmation_seed": int(confirmation_seed),
        "search_report": report(search_run, seed=SEARCH_SEED, target_id=target_id),
        "confirmation_report": report(confirmation_run, seed=confirmation_seed, target_id=target_id),
    })


def verify_subject(doc: Mapping[str, Any]) -> dict[str, Any]:
    """Recompute the verdict and digest of an archived subject; raise if either differs."""
    again = _finalize(dict(doc))
    if json.loads(_canonical(again)) != json.loads(_canonical(dict(doc))):
        raise ValueError(f"{doc.get('instance_key')}: the archived subject is not its recomputed verdict/digest")
    return again


def confirm(parent: "pp.Parent", opspec: Mapping[str, Any], points: Sequence["pp.Point"], *,
            make_inputs: Callable[["pp.Point", int], Mapping[str, Any]],
            baseline: Callable[..., Any],
            verify: Callable[["pp.Point", Mapping[str, Any], Mapping[str, Any]], tuple[bool, str]],
            master_seed: int, reps: int = 15) -> tuple[list["pp.ShardRun"], list[dict[str, Any]]]:
    """Search and confirmation runs of every point (``make_inputs(point, seed)``), both from a
    fresh nvcc build; returns the search runs (for the accounts) and the subject documents."""
    digest = pp.domain_digest(points)
    runs, subjects = [], []
    for p in points:
        base = baseline if p.usage == "benchmark" else None
        search = pp.run_point(parent, opspec, p, make_inputs(p, SEARCH_SEED), baseline=base, verify=verify, reps=reps,
                              use_cache=False)
        seed = fresh_seed(master_seed, digest, p.instance_key)
        conf = pp.run_point(parent, opspec, p, make_inputs(p, seed), baseline=base, verify=verify, reps=reps, use_cache=False)
        if p.usage == "benchmark":
            runs.append(search)
        subjects.append(subject(search, conf, confirmation_seed=seed))
    return runs, subjects


class PublicationRefused(RuntimeError):
    """Not every benchmark subject is confirmed, or the accounts are not publishable."""


def publish(catalog: str | Path, task: str, dtype: str, parent: "pp.Parent", runs: Sequence["pp.ShardRun"],
            subjects: Sequence[Mapping[str, Any]], *, target_id: str = TARGET_ID) -> Path:
    """Archive a confirmed portfolio under ``<catalog>/<target>/<task>/<dtype>/<parent sha[:16]>/``."""
    verified = [verify_subject(s) for s in subjects]
    rejected = [f"{s['instance_key']}:{s['reason']}" for s in verified if s["status"] != "confirmed"]
    if rejected:
        raise PublicationRefused(f"unconfirmed subjects: {rejected}")
    report_ = pp.performance(runs)
    if not report_.publishable:
        raise PublicationRefused(f"the accounts are not publishable: {list(report_.failure_reasons)}")
    keys = {s["instance_key"] for s in verified}
    missing = [r.point.instance_key for r in runs if r.point.instance_key not in keys]
    if missing:
        raise PublicationRefused(f"benchmark shards without a subject confirmation: {missing}")
    out = Path(catalog) / target_id / task / dtype / parent.sha256[:16]
    (out / "subjects").mkdir(parents=True, exist_ok=True)
    (out / "parent.json").write_text(parent.to_json() + "\n")
    perf = report_.document()
    perf["shards_detail"] = [{"instance_key": r.point.instance_key, "provider": r.provider, "selected": r.selected,
                              "candidate_us": r.candidate_us, "baseline_us": r.baseline_us, "candidate_cv": r.candidate_cv,
                              "attempts": r.attempts} for r in runs]
    (out / "performance.json").write_text(json.dumps(perf, indent=1, sort_keys=True) + "\n")
    digests = {}
    for s in verified:
        _, size, usage = s["instance_key"].split("/")
        (out / "subjects" / f"{size}-{usage}.json").write_text(json.dumps(s, indent=1, sort_keys=True) + "\n")
        digests[s["instance_key"]] = s["confirmation_digest"]
    manifest = {"task": task, "dtype": dtype, "target_id": target_id, "parent_sha256": parent.sha256,
                "domain_plan_digest": parent.document["domain_plan_digest"], "subjects": digests,
                "effective_end_to_end_speedup": report_.effective_end_to_end_speedup,
                "specialized_hit_speedup": report_.specialized_hit_speedup}
    (out / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    return out
