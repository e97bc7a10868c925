"""Compile and launch heartbeat hooks of an evaluation worker.

The reference's workers (tcenv/worker.py:21-55, tcenv/v2_worker.py:245-270) install two
``(begin, end)`` callback pairs through ``Backend.set_heartbeat_hooks``; the backend runs the
compile pair around every compiler run and the launch pair around every GPU launch it waits for,
and the worker's callbacks overwrite one heartbeat record that the parent ages to kill a stuck
compile or launch.  This module is that registry for the CUDA backend:

* :func:`set_compile_hooks` / :func:`set_launch_hooks` replace a pair (``None`` clears it);
* :func:`compiling` / :func:`launching` are the context managers the builder (around nvcc), the
  correctness loop (around each case's trials) and the timing loop (around each k-launch batch)
  enter; with no hooks installed they cost one tuple read.

The record is the reference's fixed-width interchange form: one stage letter (``C`` compiling,
``B`` in a launch, ``W`` queued for the GPU lock, ``E`` anything else), the wall-clock time as
``%020.6f`` and a newline, 22 bytes written in place at offset 0, so a reader never sees a
longer, older record behind a shorter new one.
"""

from __future__ import annotations

import os
import time
from contextlib import contextmanager
from pathlib import Path
from typing import Callable, Iterator

RECORD_BYTES = 22

Hook = Callable[[], object]
_compile: tuple[Hook | None, Hook | None] = (None, None)
_launch: tuple[Hook | None, Hook | None] = (None, None)


def set_compile_hooks(begin: Hook | None, end: Hook | None) -> None:
    global _compile
    _compile = (begin, end)


def set_launch_hooks(begin: Hook | None, end: Hook | None) -> None:
    global _launch
    _launch = (begin, end)


@contextmanager
def _bracket(pair: tuple[Hook | None, Hook | None]) -> Iterator[None]:
    begin, end = pair
    if begin is not None:
        begin()
    try:
        yield
    finally:
        if end is not None:
            end()


def compiling():
    return _bracket(_compile)


def launching():
    return _bracket(_launch)


def record(stage: str, at: float | None = None) -> bytes:
    """The 22-byte record of ``stage`` (one letter) at ``at`` (default: now)."""
    if len(stage) != 1:
        raise ValueError(f"a heartbeat stage is one letter, got {stage!r}")
    out = f"{stage}{time.time() if at is None else at:020.6f}\n".encode("ascii")
    if len(out) != RECORD_BYTES:
        raise ValueError(f"heartbeat time {at!r} does not fit the record")
    return out


def parse(raw: bytes) -> tuple[str, float] | None:
    """``(stage, time)`` of a record, or None for a missing or half-written one (no beat)."""
    if len(raw) < RECORD_BYTES:
        return None
    try:
        text = raw[:RECORD_BYTES].decode("ascii")
        if not text[0].isalpha() or text[-1] != "\n":
            return None
        return text[0], float(text[1:-1])
    except (UnicodeDecodeError, ValueError):
        return None


class HeartbeatFile:
    """The worker's writer: ``mark("B")`` overwrites the record in place."""

    def __init__(self, path: str | Path) -> None:
        self.path = Path(path)
        self._fd = os.open(self.path, os.O_WRONLY | os.O_CREAT, 0o600)

    def mark(self, stage: str) -> None:
        os.pwrite(self._fd, record(stage), 0)

    def install(self) -> None:
        """Route the compile, launch and GPU-lock waits of this process to this file."""
        from . import gpulock

        set_compile_hooks(lambda: self.mark("C"), lambda: self.mark("E"))
        set_launch_hooks(lambda: self.mark("B"), lambda: self.mark("E"))
        gpulock.set_wait_hooks(lambda: self.mark("W"), lambda: self.mark("E"))

    def close(self) -> None:
        os.close(self._fd)


def read(path: str | Path) -> tuple[str, float] | None:
    try:
        return parse(Path(path).read_bytes())
    except OSError:
        return None
