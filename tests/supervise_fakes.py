"""Fake worker callables for the supervision tests: every failure is made on the host (a sleep
under a launch or compile heartbeat, an exit without a report, an exception), never on a GPU."""

from __future__ import annotations

import os
import time


def ok(heartbeat, value=1):
    heartbeat.mark("B")
    heartbeat.mark("E")
    return {"status": "ok", "value": value}


def hang_in_launch(heartbeat, seconds=60.0):
    heartbeat.mark("B")
    time.sleep(seconds)
    return {"status": "ok"}


def slow_compile(heartbeat, seconds=60.0):
    heartbeat.mark("C")
    time.sleep(seconds)
    return {"status": "ok"}


def queued_then_done(heartbeat, queued=1.5, work=0.2):
    heartbeat.mark("W")
    time.sleep(queued)
    heartbeat.mark("E")
    time.sleep(work)
    return {"status": "ok"}


def busy(heartbeat, seconds=60.0):
    heartbeat.mark("E")
    time.sleep(seconds)
    return {"status": "ok"}


def exits_without_report(heartbeat):
    os._exit(3)


def raises(heartbeat):
    raise ValueError("candidate blew up")


def holds_lock_then_hangs(heartbeat, lock_dir, device=7):
    os.environ["SF_GPU_LOCK_DIR"] = lock_dir
    from shapeforge_b200 import gpulock

    with gpulock.gpu_lock("timing", device=device):
        heartbeat.mark("B")
        time.sleep(60.0)
    return {"status": "ok"}


def builds_a_candidate(heartbeat, source):
    """Compile a candidate with the track builder (fresh nvcc run): it marks C around nvcc."""
    from shapeforge_b200.track_factory import CudaTrackBuilder

    build = CudaTrackBuilder().build(source, use_cache=False)
    return {"status": "ok", "kernels": list(build.kernels), "cache_hit": build.cache_hit}
