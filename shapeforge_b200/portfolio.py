"""Shape portfolios: exact one-of-N dispatch with a declared fallback, and the two accounts.

Dispatch follows the order of tcenv/portfolio/dispatch.py:1-23 and :675-720 — every guard is
evaluated, a guard error is ``dispatch_unknown``, more than one match is ``dispatch_overlap`` (no
ranking), exactly one match selects that candidate variant, zero matches select the declared
fallback (reason ``outside_candidate_coverage``) or ``dispatch_unmatched``; a request outside the
supported domain is ``unsupported_contract_capability`` and never falls back.  On the B200 the
candidate variants are the specialised kernels (tcgen05 / vectorised) and the fallback is the
general kernel of the same operator (``sf_op_desc.variant`` 1 and 2).

The accounts restate tcenv/portfolio_performance/performance.py:18-221: per-shard
``latency_ratio = candidate_us / baseline_us`` gated at 1.10, ``specialized_hit`` = median
ratio over candidate-provided shards, ``effective_end_to_end`` = sum(candidate_us) /
sum(baseline_us) over every benchmark shard (fallback included), and the fallback time / count
fractions.
"""

from __future__ import annotations

import math
import statistics
from dataclasses import dataclass, field
from typing import Any, Callable, Iterable, Mapping

MAX_REGRESSION_RATIO = 1.10
USAGES = frozenset({"benchmark", "golden"})


class ContractError(ValueError):
    """An invalid measurement or portfolio declaration (TaskContractError in the reference)."""


# ---- exact dispatch ------------------------------------------------------------------------------


@dataclass(frozen=True)
class Variant:
    name: str
    guard: Callable[[Mapping[str, Any]], bool]
    variant: int = 1  # sf_op_desc.variant of the specialised kernel


@dataclass(frozen=True)
class Fallback:
    name: str
    handles: tuple[str, ...] = ("outside_candidate_coverage",)
    variant: int = 2  # sf_op_desc.variant of the general kernel


@dataclass(frozen=True)
class DispatchRecord:
    outcome: str  # candidate | fallback | dispatch_overlap | dispatch_unmatched | dispatch_unknown | unsupported_contract_capability
    provider: str | None  # "candidate" | "fallback" | None
    selected: str | None
    variant: int | None
    detail: str = ""
    guards: tuple[tuple[str, str], ...] = ()

    @property
    def ok(self) -> bool:
        return self.provider is not None


@dataclass
class Portfolio:
    """Variants with disjoint guards over a request's named symbols, plus an optional fallback."""

    variants: tuple[Variant, ...]
    fallback: Fallback | None = None
    domain: Callable[[Mapping[str, Any]], bool] = lambda names: True

    def resolve(self, names: Mapping[str, Any]) -> DispatchRecord:
        try:
            in_domain = bool(self.domain(names))
        except Exception as exc:  # noqa: BLE001 - a broken domain check is an unknown, not a crash
            return DispatchRecord("dispatch_unknown", None, None, None, f"domain check failed: {exc}")
        if not in_domain:
            return DispatchRecord("unsupported_contract_capability", None, None, None, "request outside the supported domain")
        guards: list[tuple[str, str]] = []
        hits: list[Variant] = []
        unknown: list[str] = []
        for v in self.variants:
            try:
                hit = bool(v.guard(names))
            except Exception as exc:  # noqa: BLE001
                guards.append((v.name, "unknown"))
                unknown.append(f"{v.name}: {exc}")
                continue
            guards.append((v.name, "true" if hit else "false"))
            if hit:
                hits.append(v)
        if unknown:
            return DispatchRecord("dispatch_unknown", None, None, None, "; ".join(unknown), tuple(guards))
        if len(hits) > 1:
            return DispatchRecord("dispatch_overlap", None, None, None, ", ".join(h.name for h in hits), tuple(guards))
        if len(hits) == 1:
            return DispatchRecord("candidate", "candidate", hits[0].name, hits[0].variant, "", tuple(guards))
        reason = "outside_candidate_coverage"
        if self.fallback is not None and reason in self.fallback.handles:
            return DispatchRecord("fallback", "fallback", self.fallback.name, self.fallback.variant, reason, tuple(guards))
        return DispatchRecord("dispatch_unmatched", None, None, None, reason, tuple(guards))


# ---- accounts ------------------------------------------------------------------------------------


def _ratio(value: Any, where: str) -> float:
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise ContractError(f"{where} must be a finite positive number")
    v = float(value)
    if not math.isfinite(v) or v <= 0.0:
        raise ContractError(f"{where} must be a finite positive number")
    return v


@dataclass(frozen=True)
class ShardMeasurement:
    """One shard's measured times (performance.py:50-108): ``instance_key`` is ``task/size/usage``."""

    instance_key: str
    usage: str
    provider: str
    candidate_us: float
    baseline_us: float | None
    timing_uncertain: bool = False
    correctness_ok: bool = True
    dispatch_ok: bool = True
    unknown: bool = False

    def __post_init__(self) -> None:
        parts = self.instance_key.split("/") if isinstance(self.instance_key, str) else []
        if len(parts) != 3 or self.usage != parts[2]:
            raise ContractError("measurement usage is not the instance_key's usage")
        if self.usage not in USAGES:
            raise ContractError(f"unknown measurement usage {self.usage!r}")
        if self.provider not in ("candidate", "fallback"):
            raise ContractError("measurement provider must be candidate or fallback")
        _ratio(self.candidate_us, f"{self.instance_key}.candidate_us")
        if self.baseline_us is not None:
            _ratio(self.baseline_us, f"{self.instance_key}.baseline_us")
        for name in ("timing_uncertain", "correctness_ok", "dispatch_ok", "unknown"):
            if type(getattr(self, name)) is not bool:
                raise ContractError(f"{self.instance_key}.{name} must be bool")

    @property
    def benchmark(self) -> bool:
        return self.usage == "benchmark"

    @property
    def latency_ratio(self) -> float | None:
        return None if self.baseline_us is None else self.candidate_us / self.baseline_us

    @property
    def specialized_latency_ratio(self) -> float | None:
        return self.latency_ratio if self.provider == "candidate" else None


@dataclass(frozen=True)
class ShardVerdict:
    measurement: ShardMeasurement
    status: str
    reason: str | None

    @property
    def ok(self) -> bool:
        return self.status == "ok"


@dataclass(frozen=True)
class PerformanceReport:
    verdicts: tuple[ShardVerdict, ...]
    specialized_hit_speedup: float | None
    effective_end_to_end_speedup: float | None
    specialized_hit_latency_ratio: float | None
    effective_end_to_end_latency_ratio: float | None
    specialized_geomean_latency_ratio: float | None
    effective_geomean_latency_ratio: float | None
    fallback_time_fraction: float | None
    fallback_count_fraction: float | None
    publishable: bool
    failure_reasons: tuple[str, ...] = field(default_factory=tuple)

    @classmethod
    def evaluate(cls, measurements: Iterable[ShardMeasurement], *, expected_benchmark_keys: Iterable[str] | None = None) -> "PerformanceReport":
        rows = tuple(measurements)
        if not rows:
            raise ContractError("a performance report needs at least one measurement")
        keys = [r.instance_key for r in rows]
        if len(set(keys)) != len(keys):
            raise ContractError("duplicate performance measurement instance_key")
        bench = [r for r in rows if r.benchmark]
        if not bench:
            raise ContractError("golden-only measurements cannot enter performance comparison")
        failures: list[str] = []
        if expected_benchmark_keys is not None:
            expected = set(expected_benchmark_keys)
            actual = {r.instance_key for r in bench}
            if expected - actual:
                failures.append(f"missing_shards:{sorted(expected - actual)}")
            if actual - expected:
                failures.append(f"unexpected_shards:{sorted(actual - expected)}")
        verdicts: list[ShardVerdict] = []
        for r in rows:
            if not r.benchmark:
                verdicts.append(ShardVerdict(r, "ignored_golden", None))
                continue
            reason = None
            if r.unknown:
                reason = "unknown"
            elif r.timing_uncertain:
                reason = "timing_uncertain"
            elif not r.correctness_ok:
                reason = "correctness_failed"
            elif not r.dispatch_ok:
                reason = "dispatch_failed"
            elif r.baseline_us is None:
                reason = "missing_baseline"
            if reason is not None:
                failures.append(f"{r.instance_key}:{reason}")
            verdicts.append(ShardVerdict(r, "ok" if reason is None else "rejected", reason))
        for r in bench:
            if r.latency_ratio is not None and r.latency_ratio > MAX_REGRESSION_RATIO:
                failures.append(f"{r.instance_key}:effective_ratio>{MAX_REGRESSION_RATIO:.2f}")
            if r.specialized_latency_ratio is not None and r.specialized_latency_ratio > MAX_REGRESSION_RATIO:
                failures.append(f"{r.instance_key}:specialized_ratio>{MAX_REGRESSION_RATIO:.2f}")
        specialized = [r for r in bench if r.provider == "candidate" and r.baseline_us is not None]
        if not specialized:
            failures.append("no_specialized_variant")
        if failures:
            return cls(tuple(verdicts), None, None, None, None, None, None, None, None, False, tuple(failures))
        spec_ratio = float(statistics.median(r.specialized_latency_ratio for r in specialized))
        eff_ratio = _ratio(sum(r.candidate_us for r in bench) / sum(r.baseline_us for r in bench), "effective_end_to_end_latency_ratio")
        spec_geo = math.exp(statistics.fmean(math.log(r.specialized_latency_ratio) for r in specialized))
        eff_geo = math.exp(statistics.fmean(math.log(r.latency_ratio) for r in bench))
        fb_time = sum(r.candidate_us for r in bench if r.provider == "fallback")
        total = sum(r.candidate_us for r in bench)
        return cls(
            verdicts=tuple(verdicts),
            specialized_hit_speedup=1.0 / spec_ratio,
            effective_end_to_end_speedup=1.0 / eff_ratio,
            specialized_hit_latency_ratio=spec_ratio,
            effective_end_to_end_latency_ratio=eff_ratio,
            specialized_geomean_latency_ratio=spec_geo,
            effective_geomean_latency_ratio=eff_geo,
            fallback_time_fraction=fb_time / total,
            fallback_count_fraction=sum(r.provider == "fallback" for r in bench) / len(bench),
            publishable=True,
        )

    def document(self) -> dict:
        return {
            "specialized_hit_speedup": self.specialized_hit_speedup,
            "effective_end_to_end_speedup": self.effective_end_to_end_speedup,
            "specialized_hit_latency_ratio": self.specialized_hit_latency_ratio,
            "effective_end_to_end_latency_ratio": self.effective_end_to_end_latency_ratio,
            "fallback_time_fraction": self.fallback_time_fraction,
            "fallback_count_fraction": self.fallback_count_fraction,
            "publishable": self.publishable,
            "failure_reasons": list(self.failure_reasons),
            "shards": [
                {"instance_key": v.measurement.instance_key, "provider": v.measurement.provider, "status": v.status,
                 "reason": v.reason, "candidate_us": v.measurement.candidate_us, "baseline_us": v.measurement.baseline_us}
                for v in self.verdicts
            ],
        }


# ---- the B200 portfolios of the workloads ----------------------------------------------------------

def gemm_nt_portfolio() -> Portfolio:
    """tcgen05 variant for TMA-legal shapes (K % 8 == 0), general fallback otherwise."""
    return Portfolio(
        variants=(Variant("gemm_nt.tcgen05_128x256", lambda n: n["K"] % 8 == 0 and n["K"] > 0 and n["aligned"]),),
        fallback=Fallback("gemm_nt.general"),
        domain=lambda n: n["M"] >= 0 and n["N"] >= 0 and n["K"] >= 0,
    )


def rmsnorm_portfolio() -> Portfolio:
    return Portfolio(
        variants=(Variant("rmsnorm.vec16B_row_in_registers", lambda n: n["H"] % 8 == 0 and n["H"] <= 65536 and n["aligned"]),),
        fallback=Fallback("rmsnorm.general_two_pass"),
        domain=lambda n: n["M"] >= 0 and n["H"] >= 1,
    )


def attention_portfolio() -> Portfolio:
    return Portfolio(
        variants=(Variant("attention.tcgen05_d64_d128", lambda n: n["D"] in (64, 128) and n["aligned"]),),
        fallback=Fallback("attention.general_warp_per_row"),
        domain=lambda n: n["D"] <= 256 and n["S"] >= 0,
    )
