"""Host-side harness logic (no GPU): fill plans, timing protocol, exact dispatch, accounts, the
Backend protocol's text hooks, and the drop-in through the reference's own loaders."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

from shapeforge_b200 import compare, portfolio, protocol, runtime
from shapeforge_b200.backend import CudaBackend, LaunchStage

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))


# ---- fill plans (tcenv/track/protocol.py:107-143) --------------------------------------------------

def test_fill_plan_matches_reference_protocol():
    import torch

    specs = [runtime.TensorSpec("x", (4,), torch.float16, "input"), runtime.TensorSpec("y", (4,), torch.float16, "output"),
             runtime.TensorSpec("ws", (8,), torch.float32, "workspace"), runtime.TensorSpec("st", (2,), torch.float32, "read_write")]
    p1, p2, p3 = (runtime.fill_plan(specs, t) for t in runtime.TRIALS)
    assert p1 == p3 == {"x": runtime.RESTORE, "y": runtime.POISON, "ws": runtime.POISON, "st": runtime.RESTORE}
    assert p2 == {"x": runtime.RESTORE, "y": runtime.ZERO, "ws": runtime.ZERO, "st": runtime.RESTORE}
    with pytest.raises(ValueError):
        runtime.fill_plan(specs, "out4")
    assert (runtime.GUARD_PATTERN, runtime.GUARD_BYTES, runtime.POISON_PATTERN) == (0xCD, 16384, 0xFF)


def test_fill_plan_agrees_with_reference_module():
    if not REF.is_dir():
        pytest.skip("reference checkout not mounted")
    sys.path.append(str(REF))  # after this repository: the reference also has a `tests` package
    from tcenv.track import protocol as ref_protocol

    assert ref_protocol.GUARD_PATTERN == runtime.GUARD_PATTERN
    assert ref_protocol.GUARD_BYTES == runtime.GUARD_BYTES
    assert ref_protocol.POISON_PATTERN == runtime.POISON_PATTERN
    assert tuple(ref_protocol.CORRECTNESS_TRIALS) == runtime.TRIALS


# ---- comparator (testing.py:140-177) -----------------------------------------------------------------

def test_scaled_error_specials_and_floor():
    ref = np.array([1.0, np.nan, np.inf, -np.inf, 0.0])
    ok = np.array([1.001, np.nan, np.inf, -np.inf, 0.0])
    assert compare.check(ok, ref, 1.0, rtol=2e-3, atol_rel=1e-3, dtype="fp16").ok
    for bad in ([1.0, 0.0, np.inf, -np.inf, 0.0], [1.0, np.nan, -np.inf, -np.inf, 0.0], [1.0, np.nan, np.inf, -np.inf, np.nan]):
        assert not compare.check(np.array(bad), ref, 1.0, rtol=2e-3, atol_rel=1e-3, dtype="fp16").ok
    # A non-finite scale fails everything; exact means bit equality.
    assert not compare.check(ok, ref, np.nan, rtol=1, atol_rel=1).ok
    assert np.isinf(compare.scaled_error(np.array([1, 2]), np.array([1, 3]), 0, 0, 0, True)).sum() == 1
    assert compare.floor_for("fp16") == pytest.approx(0.51 * 2.0**-24)


def _reference_comparator():
    """``scaled_error`` and ``_floor`` from the reference's tcenv/backends/metal/testing.py:140-177.

    That module imports the Metal runtime at the top, so the two functions are taken out of its
    source with ``ast`` and run as written, with torch and the reference's own subnormal table
    (tcenv/dtypes.py) as their globals."""
    import ast

    import torch

    sys.path.append(str(REF))  # after this repository: the reference also has a `tests` package
    from tcenv.dtypes import FLOAT_TINY_SUBNORMAL

    path = REF / "tcenv" / "backends" / "metal" / "testing.py"
    tree = ast.parse(path.read_text())
    funcs = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in ("scaled_error", "_floor")]
    assert len(funcs) == 2
    ns = {"torch": torch, "FLOAT_TINY_SUBNORMAL": FLOAT_TINY_SUBNORMAL}
    exec(compile(ast.Module(body=funcs, type_ignores=[]), str(path), "exec"), ns)
    return ns["scaled_error"], ns["_floor"]


def test_comparator_agrees_with_reference():
    """compare.scaled_error / floor_for against the reference's own functions: random values,
    per-element and scalar scales, every dtype floor, planted specials (matching and mismatching
    NaN / +-inf), non-finite scales and exact mode; errors and pass/fail verdicts must agree."""
    if not REF.is_dir():
        pytest.skip("reference checkout not mounted")
    import torch

    ref_scaled_error, ref_floor = _reference_comparator()
    for dt in ("fp16", "bf16", "fp32", "fp64", "i32"):
        assert compare.floor_for(dt) == ref_floor(dt), dt
    rng = np.random.default_rng(0)
    specials = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 1e-8, 6e-8])

    def agree(o, r, scale, rtol, atol_rel, exact, floor):
        ours = compare.scaled_error(o, r, scale, rtol, atol_rel, exact, floor)
        sc = torch.tensor(scale) if isinstance(scale, np.ndarray) else scale
        theirs = ref_scaled_error(torch.tensor(o), torch.tensor(r), sc, rtol, atol_rel, exact, floor).numpy()
        assert ours.shape == theirs.shape
        assert np.array_equal(np.isinf(ours), np.isinf(theirs))
        assert np.array_equal(np.isnan(ours), np.isnan(theirs))
        fin = np.isfinite(ours)
        np.testing.assert_allclose(ours[fin], theirs[fin], rtol=1e-12, atol=0)
        assert np.array_equal(ours > 1.0, theirs > 1.0)

    for trial in range(40):
        n = int(rng.integers(1, 300))
        r = rng.normal(size=n) * 10.0 ** rng.integers(-6, 4)
        o = r + rng.normal(size=n) * 10.0 ** rng.integers(-8, 0)
        if trial % 2:
            idx = rng.integers(0, n, size=max(1, n // 10))
            r[idx] = rng.choice(specials, size=idx.size)
            o[idx] = np.where(rng.random(idx.size) < 0.6, r[idx], rng.choice(specials, size=idx.size))
        scale = np.abs(rng.normal(size=n)) if trial % 3 == 0 else float(abs(rng.normal()))
        dtype = ("fp16", "bf16", "fp32")[trial % 3]
        rtol, atol_rel = [(2e-3, 1e-3), (1.6e-2, 8e-3), (1e-5, 1e-6)][trial % 3]
        agree(o, r, scale, rtol, atol_rel, False, compare.floor_for(dtype))
        agree(o, r, scale, rtol, atol_rel, True, 0.0)
    # Non-finite scales fail everything, scalar or per element.
    o = rng.normal(size=16)
    for bad in (np.nan, np.inf):
        agree(o, o.copy(), bad, 2e-3, 1e-3, False, 0.0)
        sc = np.ones(16)
        sc[3] = bad
        agree(o, o.copy(), sc, 2e-3, 1e-3, False, 0.0)
    # Zero scale and zero reference: only the floor is left.
    agree(np.array([0.0, 1e-8, 3e-8, -1e-7]), np.zeros(4), 0.0, 2e-3, 1e-3, False, compare.floor_for("fp16"))


# ---- timing protocol (tcenv/bench.py) ----------------------------------------------------------------

def test_device_batch_size_targets_batch_duration():
    per = 1e-5
    k = protocol.batch_size(lambda k: k * per, target_s=0.015, kmin=4)
    assert k in (1499, 1500)  # 0.015 / 1e-5 in floating point
    assert protocol.batch_size(lambda k: k * 0.5, target_s=0.015, kmin=4) == 3  # slow: bounded by the watchdog share
    assert protocol.batch_size(lambda k: k * 1e-9, target_s=0.015, kmin=4, kmax=4000) == 4000
    assert protocol.batch_size(lambda k: k * 0.01, target_s=0.015, kmin=4) == 4  # at least the rotating sets
    # The doubling search never runs a batch near the watchdog share.
    sizes = []
    protocol.batch_size(lambda k: sizes.append(k) or k * 0.2, target_s=0.015, kmin=4)
    assert max(sizes) == 1


def test_device_protocol_rotation_and_attempts():
    firsts = []

    def runner(name, per, jitter=()):
        calls = []

        def run_k(k):
            calls.append(k)
            firsts.append(name)
            j = jitter[len(calls) % len(jitter)] if jitter else 0.0
            return per * k * (1.0 + j)
        return run_k

    noise, stats, attempts = protocol.measure_interleaved({"candidate": runner("c", 2e-6), "torch": runner("t", 3e-6)}, reps=6,
                                                          provider="device")
    assert attempts == 1 and noise == 0.0
    assert stats["candidate"].median_s == pytest.approx(2e-6)
    assert stats["torch"].reps == 6
    # Rotated order: after batch sizing, repetition r starts with runner r mod 2.
    timed = firsts[-16:]
    assert timed[0::2] == ["c", "t"] * 4
    # A runner that is always noisy: three attempts, the least noisy kept and reported.
    noisy = runner("n", 1e-5, jitter=(0.0, 0.5, -0.3))
    noise, stats, attempts = protocol.measure_interleaved({"candidate": noisy}, reps=5, provider="device")
    assert attempts == protocol.BENCH_ATTEMPTS and noise > protocol.NOISY_CV
    # candidate_serial never decides quietness.
    noise, stats, attempts = protocol.measure_interleaved({"candidate": runner("c", 2e-6), "candidate_serial": noisy}, reps=5,
                                                          provider="device")
    assert attempts == 1 and noise == 0.0


def test_harness_provider_is_the_reference_protocol():
    if not REF.is_dir():
        pytest.skip("reference checkout not mounted")
    sys.path.append(str(REF))  # after this repository: the reference also has a `tests` package
    from tcenv import bench as ref_bench

    assert protocol.harness_bench() is ref_bench
    assert (ref_bench.QUIET_CV, ref_bench.BENCH_ATTEMPTS, ref_bench.BATCH_WALL_BUDGET_S) == (
        protocol.QUIET_CV, protocol.BENCH_ATTEMPTS, protocol.BATCH_WALL_BUDGET_S)
    seen = []

    def run_k(k):
        seen.append(k)
        return 1e-5 * k

    noise, stats, attempts = protocol.measure_interleaved({"candidate": run_k}, reps=4, provider="harness")
    # The harness sizes the batch from its own probe (1, 1, then a probe batch): 0.015 / 1e-5.
    assert seen[:2] == [1, 1] and stats["candidate"].iters == ref_bench.choose_iters(lambda k: 1e-5 * k)
    assert stats["candidate"].median_s == pytest.approx(1e-5) and attempts == 1
    # The two providers agree on a deterministic runner.
    _, dev, _ = protocol.measure_interleaved({"candidate": run_k}, reps=4, provider="device")
    assert dev["candidate"].median_s == pytest.approx(stats["candidate"].median_s)


# ---- exact dispatch and accounts -----------------------------------------------------------------------

def test_exact_dispatch_outcomes():
    p = portfolio.gemm_nt_portfolio()
    r = p.resolve({"M": 4096, "N": 4096, "K": 4096, "aligned": True})
    assert (r.outcome, r.provider, r.variant) == ("candidate", "candidate", 1)
    r = p.resolve({"M": 64, "N": 64, "K": 60, "aligned": True})
    assert (r.outcome, r.provider, r.variant) == ("fallback", "fallback", 2)
    assert r.detail == "outside_candidate_coverage"
    assert p.resolve({"M": -1, "N": 4, "K": 8, "aligned": True}).outcome == "unsupported_contract_capability"
    overlap = portfolio.Portfolio((portfolio.Variant("a", lambda n: True), portfolio.Variant("b", lambda n: True)))
    assert overlap.resolve({}).outcome == "dispatch_overlap"
    unknown = portfolio.Portfolio((portfolio.Variant("a", lambda n: n["missing"] > 0),), portfolio.Fallback("f"))
    assert unknown.resolve({}).outcome == "dispatch_unknown"
    assert portfolio.Portfolio((portfolio.Variant("a", lambda n: False),)).resolve({}).outcome == "dispatch_unmatched"


def _m(key, provider, cand, base, **kw):
    return portfolio.ShardMeasurement(key, key.split("/")[2], provider, cand, base, **kw)


def test_accounts_specialized_and_effective():
    rows = [_m("gemm/4096/benchmark", "candidate", 100.0, 120.0), _m("gemm/512/benchmark", "candidate", 8.0, 10.0),
            _m("gemm/odd/benchmark", "fallback", 50.0, 50.0), _m("gemm/small/golden", "candidate", 1.0, 1.0)]
    rep = portfolio.PerformanceReport.evaluate(rows)
    assert rep.publishable
    assert rep.specialized_hit_latency_ratio == pytest.approx(np.median([100 / 120, 8 / 10]))
    assert rep.effective_end_to_end_latency_ratio == pytest.approx(158.0 / 180.0)
    assert rep.fallback_count_fraction == pytest.approx(1 / 3)
    assert rep.fallback_time_fraction == pytest.approx(50 / 158)
    slow = portfolio.PerformanceReport.evaluate(rows + [_m("gemm/big/benchmark", "candidate", 120.0, 100.0)])
    assert not slow.publishable and any("ratio>1.10" in f for f in slow.failure_reasons)
    with pytest.raises(portfolio.ContractError):
        _m("gemm/x/benchmark", "other", 1.0, 1.0)


def test_accounts_agree_with_reference():
    if not REF.is_dir():
        pytest.skip("reference checkout not mounted")
    sys.path.append(str(REF))  # after this repository: the reference also has a `tests` package
    from tcenv.portfolio_performance import performance as ref_perf

    spec = [("t/a/benchmark", "candidate", 10.0, 12.0), ("t/b/benchmark", "fallback", 5.0, 4.8), ("t/c/benchmark", "candidate", 3.0, 3.3)]
    ours = portfolio.PerformanceReport.evaluate([_m(*s) for s in spec])
    theirs = ref_perf.PerformanceReport.evaluate([ref_perf.ShardMeasurement(k, k.split("/")[2], p, c, b) for k, p, c, b in spec])
    for name in ("specialized_hit_speedup", "effective_end_to_end_speedup", "fallback_time_fraction", "fallback_count_fraction",
                 "publishable"):
        assert getattr(ours, name) == pytest.approx(getattr(theirs, name)), name


# ---- Backend protocol text hooks --------------------------------------------------------------------

def test_backend_text_hooks():
    b = CudaBackend()
    assert (b.id, b.version, b.file_ext, b.language) == ("cuda-sm100", "1", ".cu", "cuda")
    src = 'extern "C" __global__ void k(const __half* x, __half* y) {}\n/* taic-launch\nkernel k grid=64,2 threads=256 smem=1024\n*/'
    stages = b.parse_launch(src)
    assert stages == [LaunchStage("k", (64, 2, 1), (256, 1, 1), 1024)]
    assert b.validate_launch(stages, {"max_threads_per_threadgroup": 1024, "max_threadgroup_memory_bytes": 232448}) == []
    assert b.validate_launch([LaunchStage("k", (1, 1, 1), (2048, 1, 1))], {}) != []
    assert b.screen(src) == []
    assert b.screen(src + "\nvoid f(){ __trap(); }")
    assert b.device_matches({"match_name_contains": "B200"}, {"name": "NVIDIA B200", "cc_major": 10})
    assert not b.device_matches({"match_name_contains": "B200"}, {"name": "NVIDIA H100", "cc_major": 9})
    cal = b.calibration("b200")
    roof = b.roofline({"min_bytes": 67117056, "flops": 4 * 4096 * 4096, "dtype": "fp16"}, 12.8e-6, cal)
    assert roof["bound"] == "memory"
    assert roof["bandwidth_fraction"] == pytest.approx(67117056 / 12.8e-6 / (cal["copy_gbs"] * 1e9))
    assert "const __half* __restrict__ x" in b.abi_stub({"tensors": [{"name": "x", "dtype": "fp16", "access": "read"}]})


def test_plugin_loads_through_reference_registry_and_target():
    """The drop-in: the reference's own load_backend / load_target resolve cuda-sm100 / b200."""
    if not REF.is_dir():
        pytest.skip("reference checkout not mounted")
    sys.path.append(str(REF))  # after this repository: the reference also has a `tests` package
    import tcenv.backends.registry as registry
    import tcenv.target as target

    from shapeforge_b200 import bootstrap

    saved = (registry.BACKENDS, target.BACKENDS, target.TARGETS)
    try:
        bootstrap.install()
        b = registry.load_backend("cuda-sm100")
        assert isinstance(b, CudaBackend) and b.version == "1"
        prof = target.load_target("b200")
        assert prof.backend == "cuda-sm100" and prof.status == "active"
        assert int(prof.raw_limits["max_threadgroup_memory_bytes"]) == 232448
        from tcenv.track.abi import REQUIRED_TARGET_LIMITS

        assert set(REQUIRED_TARGET_LIMITS) <= set(prof.raw_limits)
    finally:
        registry.BACKENDS, target.BACKENDS, target.TARGETS = saved
        registry.load_backend.cache_clear()


def test_track_registry_file_loads_with_reference_loader():
    if not REF.is_dir():
        pytest.skip("reference checkout not mounted")
    sys.path.append(str(REF))  # after this repository: the reference also has a `tests` package
    from tcenv.track.registry import load_track_registry

    reg = load_track_registry(ROOT / "backends" / "cuda-sm100" / "tracks.json")
    assert "cuda-single" in {t.track_id for t in reg.tracks}
