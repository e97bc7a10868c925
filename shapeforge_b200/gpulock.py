"""Per-device GPU lock: no measurement on a GPU overlaps other GPU work this project starts on it.

The reference keeps one machine-wide lock (tcenv/gpulock.py: ``gpu_lock(what, exclusive=...)``,
``flock(2)`` on one file, exclusive for timing, shared for untimed GPU work, re-entrant, upgrades
release the shared hold first).  A B200 node has eight GPUs and one worker per GPU, so the lock is
keyed by device index: timing on GPU 3 excludes other work on GPU 3 only.  Same rules otherwise:

* ``gpu_lock(what, exclusive=True)`` for timing, ``exclusive=False`` for compilation and
  correctness; yields the seconds spent waiting;
* re-entrant in a process: inside an exclusive hold every request passes; inside a shared hold a
  shared request passes and an exclusive one upgrades for its block (releasing the shared hold
  first — two holders upgrading while still sharing would wait on each other forever) and then
  returns to shared;
* the lock is ``flock`` on ``<dir>/gpu<index>.lock``, so the kernel releases it when the holder
  exits, killed or not; an exclusive holder writes its pid and purpose into the file
  (``holder(device)``); ``<index>`` is the physical GPU: a process restricted by
  ``CUDA_VISIBLE_DEVICES`` (a per-GPU worker sees its GPU as device 0) locks the GPU the mask
  names, so workers on different GPUs never share a lock;
* waiting longer than ``max_wait_s`` raises ``GpuLockTimeout``; ``set_wait_hooks`` lets a worker
  mark its heartbeat while it queues.

The directory is ``$SF_GPU_LOCK_DIR`` or ``~/.cache/shapeforge_b200``.
"""

from __future__ import annotations

import fcntl
import os
import time
from contextlib import contextmanager
from pathlib import Path
from typing import Callable, Iterator

DEFAULT_MAX_WAIT_S = 1800.0
_POLL_S = 0.05


class GpuLockTimeout(RuntimeError):
    """The lock was not obtained within the caller's wait limit."""


class _State:
    def __init__(self) -> None:
        self.fd: int | None = None
        self.mode: str | None = None  # "sh" | "ex" while held
        self.what = ""
        self.writable = True


_states: dict[int | str, _State] = {}
_wait_hooks: tuple[Callable[[], None], Callable[[], None]] | None = None


def lock_dir() -> Path:
    return Path(os.environ.get("SF_GPU_LOCK_DIR") or Path.home() / ".cache" / "shapeforge_b200")


def lock_file(device: int | str) -> Path:
    return lock_dir() / f"gpu{device}.lock"


def physical_device(logical: int) -> int | str:
    """The GPU behind this process's device ``logical``: its entry of ``CUDA_VISIBLE_DEVICES``
    (an index, or a UUID / MIG name made file-name safe) when the mask is set, else ``logical``."""
    mask = os.environ.get("CUDA_VISIBLE_DEVICES")
    if mask is None or not mask.strip():
        return int(logical)
    entries = [e.strip() for e in mask.split(",") if e.strip()]
    if not 0 <= logical < len(entries):
        return int(logical)
    entry = entries[logical]
    if entry.isdigit():
        return int(entry)
    return "".join(ch if ch.isalnum() or ch in "-_" else "_" for ch in entry)


def set_wait_hooks(on_wait: Callable[[], None], on_acquired: Callable[[], None]) -> None:
    """``on_wait`` runs when the lock is found busy, ``on_acquired`` once it was obtained after waiting."""
    global _wait_hooks
    _wait_hooks = (on_wait, on_acquired)


def holder(device: int | str) -> str:
    """The exclusive holder's note (``pid N: what``), or "" when none was written."""
    try:
        return lock_file(device).read_text(encoding="utf-8", errors="replace").strip()
    except OSError:
        return ""


def _current_device() -> int:
    try:
        import torch

        if torch.cuda.is_available():
            return int(torch.cuda.current_device())
    except Exception:  # noqa: BLE001 - no CUDA runtime: device 0
        pass
    return 0


def _acquire(fd: int, flag: int, max_wait_s: float) -> float:
    t0 = time.monotonic()
    waited = False
    while True:
        try:
            fcntl.flock(fd, flag | fcntl.LOCK_NB)
            if waited and _wait_hooks:
                _wait_hooks[1]()
            return time.monotonic() - t0
        except BlockingIOError:
            if not waited:
                waited = True
                if _wait_hooks:
                    _wait_hooks[0]()
            if time.monotonic() - t0 > max_wait_s:
                raise GpuLockTimeout(f"GPU lock busy for {max_wait_s:.1f} s") from None
            time.sleep(_POLL_S)


@contextmanager
def gpu_lock(what: str, *, exclusive: bool = True, device: int | None = None,
             max_wait_s: float = DEFAULT_MAX_WAIT_S) -> Iterator[float]:
    """Hold the lock of ``device`` (this process's device index; default: the current CUDA
    device) for the block; the lock is the physical GPU's (``physical_device``)."""
    dev = physical_device(_current_device() if device is None else int(device))
    st = _states.setdefault(dev, _State())
    want = "ex" if exclusive else "sh"
    outer, outer_what = st.mode, st.what
    if outer == "ex" or outer == want:
        yield 0.0
        return
    if st.fd is None:
        path = lock_file(dev)
        try:
            path.parent.mkdir(parents=True, exist_ok=True)
            st.fd = os.open(path, os.O_RDWR | os.O_CREAT, 0o644)
            st.writable = True
        except OSError:
            st.fd = os.open(path, os.O_RDONLY)  # flock needs no write access
            st.writable = False
    if outer == "sh":
        fcntl.flock(st.fd, fcntl.LOCK_UN)  # release before upgrading
        st.mode = None
    try:
        waited = _acquire(st.fd, fcntl.LOCK_EX if exclusive else fcntl.LOCK_SH, max_wait_s)
    except BaseException:
        if outer is None:
            os.close(st.fd)
            st.fd, st.what = None, ""
        else:
            _acquire(st.fd, fcntl.LOCK_SH, max_wait_s)
            st.mode, st.what = "sh", outer_what
        raise
    st.mode, st.what = want, what
    if exclusive and st.writable:
        os.ftruncate(st.fd, 0)
        os.pwrite(st.fd, f"pid {os.getpid()}: {what}\n".encode(), 0)
    try:
        yield waited
    finally:
        if exclusive and st.writable:
            os.ftruncate(st.fd, 0)
        if outer == "sh":
            fcntl.flock(st.fd, fcntl.LOCK_UN)
            st.mode, st.what = None, ""
            _acquire(st.fd, fcntl.LOCK_SH, max_wait_s)
            st.mode, st.what = "sh", outer_what
        else:
            os.close(st.fd)  # closing the descriptor releases the lock
            st.fd, st.mode, st.what, st.writable = None, None, "", True
