"""Timing of candidate and baseline launches: per-launch medians from interleaved repetitions.

The contract every ShapeForge backend is timed by (tcenv/bench.py:65-220) is: runners are
``run_k(k) -> seconds`` for k back-to-back launches; each runner's batch size is chosen so one
batch lasts about 15 ms but never longer than the launch watchdog allows (1.6 s); every
repetition times each runner once, in varying order, after discarded warm-up repetitions; the
kept number is the median per-launch time; an attempt is quiet when the largest CV over the
runners (``candidate_serial`` excluded) is at most 0.05; at most three attempts, keeping the first
quiet one, else the least noisy.

Two providers of that contract:

* ``harness`` — inside the ShapeForge harness (``tcenv`` importable), ``measure_interleaved``
  hands the runners to the harness's own ``tcenv.bench.measure_interleaved``, so CUDA candidates
  are timed by exactly the code that times every other backend;
* ``device`` — this library used on its own: batch sizes by a doubling search over measured
  batches (1, 2, 4, ... launches until one batch passes a quarter of the target), repetitions in
  a rotated order (repetition r starts at runner r mod n, so each runner takes every position
  equally often), the same quietness rule and attempt limit.

``provider="auto"`` picks ``harness`` when ``tcenv.bench`` imports and ``device`` otherwise.  The
B200 candidate runner is ``sf_run_batch`` (device time between two CUDA events over k launches on
rotating argument sets); ``cuda_event_runner`` builds the same kind of runner from a Python launch
function (baselines, compiled candidates).
"""

from __future__ import annotations

import statistics
from dataclasses import dataclass, field
from typing import Callable, Mapping

# Contract constants (tcenv/bench.py:66, :153-157): the watchdog share of one batch, the
# quietness cutoff and the attempt limit.
BATCH_WALL_BUDGET_S = 1.6
QUIET_CV = 0.05
NOISY_CV = QUIET_CV
BENCH_ATTEMPTS = 3
# The runner that only re-measures the candidate serially never decides quietness.
NOISE_EXEMPT = ("candidate_serial",)

Runner = Callable[[int], float]


@dataclass
class BenchStats:
    """Per-launch statistics of one runner (the report's timing record)."""

    median_s: float
    mean_s: float
    min_s: float
    cv: float
    reps: int
    iters: int
    samples_s: tuple = field(default_factory=tuple)

    def to_dict(self) -> dict:
        return {
            "median_s": self.median_s,
            "mean_s": self.mean_s,
            "min_s": self.min_s,
            "cv": self.cv,
            "reps": self.reps,
            "iters": self.iters,
        }


def harness_bench():
    """The harness's timing module, or None when this library runs outside the harness."""
    try:
        from tcenv import bench
    except Exception:
        return None
    return bench


def batch_size(run_k: Runner, target_s: float = 0.015, kmin: int = 4, kmax: int = 4000) -> int:
    """Launches per timed batch so that one batch lasts about ``target_s``.

    Batches of 1, 2, 4, ... launches are timed (after one discarded launch) until a batch passes a
    quarter of the target, ``kmax`` is reached or a batch gets near the watchdog share; the last
    batch's per-launch time sizes k.  k is at least ``kmin`` (the rotating buffer sets) unless
    ``kmin`` launches would exceed the watchdog share, and never makes a batch longer than it."""
    run_k(1)  # one-time costs (module load, graph instantiation) stay out of the estimate
    k = 1
    while True:
        t = max(run_k(k), 1e-9)
        if t >= 0.25 * target_s or k >= kmax or t >= 0.25 * BATCH_WALL_BUDGET_S:
            break
        k = min(2 * k, kmax)
    per = t / k
    want = min(kmax, max(kmin, int(target_s / per)))
    return int(max(1, min(want, BATCH_WALL_BUDGET_S / per)))


def _stats(xs: list[float], iters: int) -> BenchStats:
    mean = statistics.fmean(xs)
    # A single repetition has no measurable spread: it counts as the noisiest possible, so it can
    # never pass the quietness gate on its own.
    cv = statistics.pstdev(xs) / mean if (len(xs) > 1 and mean > 0) else 1.0
    return BenchStats(statistics.median(xs), mean, min(xs), cv, len(xs), iters, tuple(xs))


def noise(stats: Mapping[str, BenchStats]) -> float:
    """Largest CV over the runners that decide whether an attempt is quiet."""
    cvs = [s.cv for name, s in stats.items() if name not in NOISE_EXEMPT]
    return max(cvs) if cvs else 0.0


def rotated_repetitions(runners: Mapping[str, Runner], *, reps: int = 15, target_s: float = 0.015, warmup_reps: int = 2,
                        kmin: int = 4, kmax: int = 4000, start: int = 0) -> dict[str, BenchStats]:
    """One attempt of the device protocol: ``warmup_reps + reps`` repetitions, each timing every
    runner once, repetition r in the runner order rotated by ``start + r``."""
    names = list(runners)
    ks = {n: batch_size(runners[n], target_s, kmin, kmax) for n in names}
    samples: dict[str, list[float]] = {n: [] for n in names}
    for r in range(warmup_reps + reps):
        shift = (start + r) % len(names)
        for n in names[shift:] + names[:shift]:
            per_launch = runners[n](ks[n]) / ks[n]
            if r >= warmup_reps:
                samples[n].append(per_launch)
    return {n: _stats(samples[n], ks[n]) for n in names}


def _from_harness(stats: Mapping[str, object]) -> dict[str, BenchStats]:
    return {n: BenchStats(s.median_s, s.mean_s, s.min_s, s.cv, s.reps, s.iters, tuple(getattr(s, "samples_s", ())))
            for n, s in stats.items()}


def measure_interleaved(runners: Mapping[str, Runner], *, reps: int = 15, seed: int = 0, kmin: int = 4,
                        attempts_max: int = BENCH_ATTEMPTS, noisy_cv: float = NOISY_CV, target_s: float = 0.015,
                        provider: str = "auto") -> tuple[float, dict[str, BenchStats], int]:
    """Time ``runners``; returns (noise of the kept attempt, per-runner stats, attempts made).

    ``provider``: ``"harness"`` (tcenv.bench, required), ``"device"`` (this module's protocol) or
    ``"auto"`` (the harness's when importable)."""
    if provider not in ("auto", "harness", "device"):
        raise ValueError(f"unknown timing provider {provider!r}")
    bench = harness_bench() if provider != "device" else None
    if provider == "harness" and bench is None:
        raise RuntimeError("the harness timing protocol (tcenv.bench) is not importable")
    if bench is not None:
        nz, stats, attempts = bench.measure_interleaved(dict(runners), reps=reps, seed=seed, kmin=kmin, attempts_max=attempts_max,
                                                        noisy_cv=noisy_cv, target_s=target_s)
        return float(nz), _from_harness(stats), int(attempts)
    kept: tuple[float, dict[str, BenchStats]] | None = None
    made = 0
    for attempt in range(attempts_max):
        stats = rotated_repetitions(runners, reps=reps, target_s=target_s, kmin=kmin, start=seed + attempt)
        made += 1
        nz = noise(stats)
        if nz <= noisy_cv:
            return float(nz), stats, made
        if kept is None or nz < kept[0]:
            kept = (nz, stats)
    assert kept is not None
    return float(kept[0]), kept[1], made


def cuda_event_runner(launch: Callable[[int], None], stream=None) -> Runner:
    """Wrap ``launch(i)`` (enqueue launch i) into ``run_k(k) -> device seconds`` using CUDA events."""
    import torch

    def run_k(k: int) -> float:
        s = stream or torch.cuda.current_stream()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(k):
            launch(i)
        e1.record(s)
        e1.synchronize()
        return e0.elapsed_time(e1) * 1e-3

    return run_k
