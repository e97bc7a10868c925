"""The per-device GPU lock on the host: exclusive excludes everything on the same device, shared
holders coexist, devices are independent, re-entrancy and upgrades behave like the reference's
machine-wide lock (tcenv/gpulock.py), and a dead holder's lock is released by the kernel.
"""

from __future__ import annotations

import multiprocessing as mp
import time

import pytest

from shapeforge_b200 import gpulock


def _hold(lock_dir, device, exclusive, ready, release, seconds):
    import os

    os.environ["SF_GPU_LOCK_DIR"] = lock_dir
    from shapeforge_b200 import gpulock as gl

    with gl.gpu_lock("child", exclusive=exclusive, device=device):
        ready.set()
        release.wait(seconds)


@pytest.fixture()
def lock_dir(tmp_path, monkeypatch):
    monkeypatch.setenv("SF_GPU_LOCK_DIR", str(tmp_path))
    return str(tmp_path)


def _child(lock_dir, device, exclusive, seconds=10.0):
    ctx = mp.get_context("spawn")
    ready, release = ctx.Event(), ctx.Event()
    p = ctx.Process(target=_hold, args=(lock_dir, device, exclusive, ready, release, seconds))
    p.start()
    assert ready.wait(60), "the child did not take the lock"
    return p, release


def test_exclusive_excludes_the_same_device_only(lock_dir):
    p, release = _child(lock_dir, 0, True)
    try:
        assert gpulock.holder(0).endswith(": child")
        with pytest.raises(gpulock.GpuLockTimeout):
            with gpulock.gpu_lock("timing", device=0, max_wait_s=0.3):
                pass
        with pytest.raises(gpulock.GpuLockTimeout):
            with gpulock.gpu_lock("correctness", exclusive=False, device=0, max_wait_s=0.3):
                pass
        with gpulock.gpu_lock("timing", device=1, max_wait_s=0.3) as waited:
            assert waited < 0.3
    finally:
        release.set()
        p.join(30)


def test_shared_holders_coexist_and_block_exclusive(lock_dir):
    p, release = _child(lock_dir, 2, False)
    try:
        with gpulock.gpu_lock("compile", exclusive=False, device=2, max_wait_s=0.3):
            pass
        with pytest.raises(gpulock.GpuLockTimeout):
            with gpulock.gpu_lock("timing", device=2, max_wait_s=0.3):
                pass
    finally:
        release.set()
        p.join(30)


def test_a_dead_holders_lock_is_released(lock_dir):
    p, release = _child(lock_dir, 3, True, seconds=60.0)
    p.kill()
    p.join(30)
    with gpulock.gpu_lock("timing", device=3, max_wait_s=5.0):
        pass


def test_reentrancy_and_upgrade(lock_dir):
    calls = []
    gpulock.set_wait_hooks(lambda: calls.append("wait"), lambda: calls.append("got"))
    try:
        with gpulock.gpu_lock("outer", device=4):
            with gpulock.gpu_lock("inner", device=4) as w1:
                with gpulock.gpu_lock("shared inside exclusive", exclusive=False, device=4) as w2:
                    assert (w1, w2) == (0.0, 0.0)
        with gpulock.gpu_lock("correctness", exclusive=False, device=4):
            with gpulock.gpu_lock("timing", device=4):
                assert gpulock.holder(4).endswith(": timing")
            # Back to shared: another process may share, not take it exclusively.
            assert gpulock._states[4].mode == "sh"
        assert gpulock._states[4].mode is None and gpulock._states[4].fd is None
        assert calls == []  # nothing ever waited
    finally:
        gpulock._wait_hooks = None


def test_wait_hooks_fire_when_queued(lock_dir):
    calls = []
    gpulock.set_wait_hooks(lambda: calls.append("wait"), lambda: calls.append("got"))
    p, release = _child(lock_dir, 5, True, seconds=0.5)
    try:
        t0 = time.monotonic()
        with gpulock.gpu_lock("timing", device=5, max_wait_s=30.0) as waited:
            assert waited > 0.0
        assert time.monotonic() - t0 < 30.0
        assert calls == ["wait", "got"]
    finally:
        gpulock._wait_hooks = None
        release.set()
        p.join(30)


def _hold_masked(lock_dir, mask, ready, release, seconds):
    import os

    os.environ["SF_GPU_LOCK_DIR"] = lock_dir
    os.environ["CUDA_VISIBLE_DEVICES"] = mask
    from shapeforge_b200 import gpulock as gl

    with gl.gpu_lock("masked child", device=0):
        ready.set()
        release.wait(seconds)


def test_lock_is_the_physical_gpu_behind_a_device_mask(lock_dir, monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "3,5")
    assert gpulock.physical_device(0) == 3 and gpulock.physical_device(1) == 5
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "GPU-1a2b/x")
    assert gpulock.physical_device(0) == "GPU-1a2b_x"
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert gpulock.physical_device(2) == 2
    # A worker that sees only GPU 3 (as its device 0) holds GPU 3's lock: device 3 here is
    # blocked, device 0 here is free.
    ctx = mp.get_context("spawn")
    ready, release = ctx.Event(), ctx.Event()
    p = ctx.Process(target=_hold_masked, args=(lock_dir, "3", ready, release, 10.0))
    p.start()
    try:
        assert ready.wait(60)
        assert gpulock.holder(3).endswith(": masked child")
        with pytest.raises(gpulock.GpuLockTimeout):
            with gpulock.gpu_lock("timing", device=3, max_wait_s=0.3):
                pass
        with gpulock.gpu_lock("timing", device=0, max_wait_s=0.3) as waited:
            assert waited < 0.3
    finally:
        release.set()
        p.join(30)
