"""Supervised evaluation on the host (tcenv/evaluate.py supervise, tcenv/v2_worker.py run_bounded_v2):
deadlines per heartbeat stage, lock waits excluded from the timeout, typed failures, and the kernel
releasing a killed worker's GPU lock.  The failures are host-made (fake workers), none on a GPU.
"""

from __future__ import annotations

import time

import pytest

from shapeforge_b200 import gpulock
from shapeforge_b200.supervise import run_bounded

F = "tests.supervise_fakes"


def test_a_finished_worker_returns_its_report():
    assert run_bounded(f"{F}:ok", {"value": 7}, timeout=60) == {"status": "ok", "value": 7}


def test_a_hung_launch_is_killed_at_the_launch_deadline():
    t0 = time.monotonic()
    rep = run_bounded(f"{F}:hang_in_launch", timeout=120, launch_deadline_s=1.0)
    assert rep["status"] == "timeout" and rep["reason"] == "launch"
    assert time.monotonic() - t0 < 30


def test_a_slow_compile_is_killed_at_the_compile_deadline():
    rep = run_bounded(f"{F}:slow_compile", timeout=120, compile_deadline_s=1.0)
    assert rep["status"] == "timeout" and rep["reason"] == "compile"


def test_the_whole_evaluation_has_a_timeout():
    rep = run_bounded(f"{F}:busy", timeout=1.0)
    assert rep["status"] == "timeout" and rep["reason"] == "timeout"


def test_time_queued_for_the_gpu_lock_does_not_count():
    rep = run_bounded(f"{F}:queued_then_done", {"queued": 2.0, "work": 0.1}, timeout=1.0)
    assert rep == {"status": "ok"}


def test_crashes_and_exceptions_are_typed():
    rep = run_bounded(f"{F}:exits_without_report", timeout=60)
    assert rep["status"] == "crash" and rep["returncode"] == 3
    rep = run_bounded(f"{F}:raises", timeout=60)
    assert rep["status"] == "runtime_error" and "candidate blew up" in rep["detail"]


def test_a_killed_workers_gpu_lock_is_released(tmp_path, monkeypatch):
    monkeypatch.setenv("SF_GPU_LOCK_DIR", str(tmp_path))
    rep = run_bounded(f"{F}:holds_lock_then_hangs", {"lock_dir": str(tmp_path)}, timeout=120, launch_deadline_s=1.0)
    assert rep["status"] == "timeout" and rep["reason"] == "launch"
    with gpulock.gpu_lock("timing", device=7, max_wait_s=5.0):
        pass


SRC = """extern "C" __global__ void k(const float* x, float* y) { y[threadIdx.x] = x[threadIdx.x]; }
/* taic-launch
kernel k grid=1 threads=32
*/
"""


def test_the_track_builder_runs_under_the_compile_deadline():
    """A real nvcc build inside a supervised worker: finishes under a generous compile deadline, and
    is killed under one shorter than nvcc's own start-up (the builder marks C around nvcc)."""
    rep = run_bounded(f"{F}:builds_a_candidate", {"source": SRC}, timeout=300, compile_deadline_s=240)
    assert rep == {"status": "ok", "kernels": ["k"], "cache_hit": False}
    rep = run_bounded(f"{F}:builds_a_candidate", {"source": SRC.replace("threadIdx.x]", "threadIdx.x] ")}, timeout=300,
                      compile_deadline_s=0.05)
    assert rep["status"] == "timeout" and rep["reason"] == "compile"


def test_heartbeat_record_is_the_fixed_width_interchange_form(tmp_path):
    from shapeforge_b200 import heartbeat

    rec = heartbeat.record("B", 1767225600.25)
    assert rec == b"B" + b"%020.6f\n" % 1767225600.25 and len(rec) == 22
    assert heartbeat.parse(rec) == ("B", 1767225600.25)
    assert heartbeat.parse(rec[:15]) is None  # half-written: no beat
    assert heartbeat.parse(b"\x00" * 22) is None
    hb = heartbeat.HeartbeatFile(tmp_path / "hb")
    hb.mark("C")
    hb.mark("E")  # overwritten in place, same width
    assert (tmp_path / "hb").stat().st_size == 22 and heartbeat.read(tmp_path / "hb")[0] == "E"
    hb.close()


def test_the_reference_parent_reads_our_worker_record(tmp_path):
    """A reference parent process supervising this backend's worker reads the same record."""
    import os
    import sys
    from pathlib import Path

    ref = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))
    if not (ref / "tcenv").is_dir():
        pytest.skip("reference checkout not mounted")
    if str(ref) not in sys.path:
        sys.path.append(str(ref))
    from tcenv.evaluate import _read_heartbeat

    from shapeforge_b200 import heartbeat

    hb = heartbeat.HeartbeatFile(tmp_path / "hb")
    hb.mark("W")
    stage, at = _read_heartbeat(tmp_path / "hb")
    assert stage == "W" and abs(at - heartbeat.read(tmp_path / "hb")[1]) < 1e-6
    hb.close()


def test_backend_hooks_bracket_nvcc_and_launches():
    """The reference's workers install (begin, end) pairs through Backend.set_heartbeat_hooks; the
    CUDA backend runs the compile pair around nvcc (not around a cache hit) and the launch pair
    around each synchronised launch."""
    from shapeforge_b200 import heartbeat
    from shapeforge_b200.backend import CudaBackend
    from shapeforge_b200.candidates import compile_source

    calls = []
    CudaBackend().set_heartbeat_hooks(on_compile=(lambda: calls.append("C"), lambda: calls.append("c")),
                                      on_launch=(lambda: calls.append("B"), lambda: calls.append("b")))
    try:
        src = 'extern "C" __global__ void hb_probe(int* x) { x[0] = 1; }\n'
        compile_source(src, name="hbprobe", use_cache=False)
        assert calls == ["C", "c"]
        compile_source(src, name="hbprobe", use_cache=True)  # served from the cache: no compiler run
        assert calls == ["C", "c"]
        with pytest.raises(RuntimeError):
            with heartbeat.launching():
                raise RuntimeError("device error")
        assert calls == ["C", "c", "B", "b"]  # the end hook runs on an error too
        CudaBackend().set_heartbeat_hooks(on_compile=None)  # an omitted pair stays installed
        with heartbeat.launching():
            pass
        assert calls[-2:] == ["B", "b"]
    finally:
        heartbeat.set_compile_hooks(None, None)
        heartbeat.set_launch_hooks(None, None)


def test_timing_batches_are_bracketed_as_launches(monkeypatch, tmp_path):
    """The portfolio shard timing and the track evaluator's timing run each synchronised k-launch
    batch inside the launch pair (a fake CUDA-event runner on the host; the real protocol)."""
    from shapeforge_b200 import heartbeat, portfolio_pack, protocol
    from shapeforge_b200.track_factory import CudaTrackEvaluator

    monkeypatch.setenv("SF_GPU_LOCK_DIR", str(tmp_path))
    inside = []
    depth = [0]
    heartbeat.set_launch_hooks(lambda: depth.__setitem__(0, depth[0] + 1), lambda: depth.__setitem__(0, depth[0] - 1))

    def fake_runner(launch, stream=None):
        def run_k(k):
            inside.append(depth[0])
            for i in range(k):
                launch(i)
            return 1e-5 * k
        return run_k

    monkeypatch.setattr(protocol, "cuda_event_runner", fake_runner)
    try:
        cand, base, noisy, attempts = portfolio_pack._timed(lambda: None, lambda: None, reps=3)
        assert inside and all(d == 1 for d in inside) and depth[0] == 0
        assert not noisy and attempts == 1 and abs(cand.median_s - 1e-5) < 1e-12

        class Runner:
            def pointers(self):
                return [0]

        inside.clear()
        doc = CudaTrackEvaluator._time(lambda ptrs: None, Runner(), 3)
        assert inside and all(d == 1 for d in inside) and depth[0] == 0
        assert doc["protocol"] == "interleaved" and doc["attempts"] == 1
    finally:
        heartbeat.set_launch_hooks(None, None)
