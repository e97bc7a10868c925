"""Build, load and launch candidate CUDA sources (the harness side of the Candidate/Harness split).

A candidate is a single CUDA source whose ``extern "C" __global__`` kernels take the task's ABI
tensors in order.  The harness compiles it for sm_100a with nvcc (``-cubin``), loads the image
through the C ABI (``sf_module_load``) and launches kernels by name (``sf_launch_kernel``).
Compiled images are cached by the hash of source + flags.
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import os
import subprocess
import tempfile
from pathlib import Path
from typing import Sequence

from . import _native, heartbeat, kernel_stats
from .build import ARCH, nvcc

CACHE = Path(os.environ.get("SF_CANDIDATE_CACHE", Path(tempfile.gettempdir()) / "shapeforge_b200_candidates"))


class CandidateCompileError(RuntimeError):
    """nvcc rejected the candidate; ``log`` holds the compiler output."""

    def __init__(self, message: str, log: str):
        super().__init__(message)
        self.log = log


def _flags(extra_flags: Sequence[str]) -> list[str]:
    return [*ARCH, "-O3", "-std=c++17", "-cubin", *extra_flags]


def cache_path(source: str, extra_flags: Sequence[str] = (), name: str = "candidate") -> Path:
    """Where the cubin of ``source`` built with ``extra_flags`` is cached (hash of source + flags)."""
    key = hashlib.sha256((source + "\0" + " ".join(_flags(extra_flags))).encode()).hexdigest()[:24]
    return CACHE / f"{name}-{key}.cubin"


def compile_source(source: str, extra_flags: Sequence[str] = (), name: str = "candidate", use_cache: bool = True) -> bytes:
    """Compile ``source`` to an sm_100a cubin and return the image bytes.  Images are cached by the
    hash of source + flags; ``use_cache=False`` always runs nvcc (a fresh build, as a confirmation
    requires) and refreshes the cached copy."""
    flags = _flags(extra_flags)
    CACHE.mkdir(parents=True, exist_ok=True)
    out = cache_path(source, extra_flags, name)
    if use_cache and out.is_file():
        return out.read_bytes()
    with tempfile.TemporaryDirectory() as d:
        src = Path(d) / f"{name}.cu"
        src.write_text(source)
        tmp = Path(d) / "out.cubin"
        with heartbeat.compiling():  # an evaluation worker's compile deadline covers nvcc only
            # -Xptxas -v only prints each entry's resources; the image is the same, so it is not
            # part of the cache key.
            proc = subprocess.run([nvcc(), *flags, "-Xptxas", "-v", str(src), "-o", str(tmp)], capture_output=True,
                                  text=True)
        if proc.returncode != 0:
            raise CandidateCompileError(f"nvcc failed for {name}", proc.stdout + proc.stderr)
        data = tmp.read_bytes()
    res = kernel_stats.parse_ptxas(proc.stdout + proc.stderr)
    _resources_path(out).write_text(json.dumps({k: v.to_dict() for k, v in res.items()}, sort_keys=True))
    out.write_bytes(data)
    return data


def _resources_path(cubin: Path) -> Path:
    return cubin.with_suffix(".resources.json")


def kernel_resources(source: str, extra_flags: Sequence[str] = (), name: str = "candidate",
                     use_cache: bool = True) -> dict[str, "kernel_stats.KernelResources"]:
    """Per-entry resources (registers, static shared memory, spills, ...) that ptxas assigned when
    ``source`` was built with ``extra_flags``; builds it when the record is missing."""
    path = _resources_path(cache_path(source, extra_flags, name))
    if not (use_cache and path.is_file() and cache_path(source, extra_flags, name).is_file()):
        compile_source(source, extra_flags, name, use_cache=False)
    doc = json.loads(path.read_text())
    return {k: kernel_stats.KernelResources(**v) for k, v in doc.items()}


class Module:
    """A loaded image; kernels are launched by name with cudaLaunchKernel argument semantics."""

    def __init__(self, image: bytes):
        self._image = ctypes.create_string_buffer(image, len(image))
        handle = ctypes.c_void_p()
        _native.call("sf_module_load", ctypes.cast(self._image, ctypes.c_void_p), len(image), ctypes.byref(handle))
        self.handle = handle
        self._functions: dict[str, ctypes.c_void_p] = {}

    def function(self, name: str) -> ctypes.c_void_p:
        if name not in self._functions:
            fn = ctypes.c_void_p()
            _native.call("sf_module_get_function", self.handle, name.encode(), ctypes.byref(fn))
            self._functions[name] = fn
        return self._functions[name]

    def launch(self, name: str, grid, block, args: Sequence[object], smem: int = 0, stream: int = 0) -> None:
        """``args``: ctypes scalars (c_int, c_float, ...) or ints (device pointers)."""
        holders = [a if isinstance(a, ctypes._SimpleCData) else ctypes.c_void_p(int(a)) for a in args]
        argv = (ctypes.c_void_p * len(holders))(*[ctypes.cast(ctypes.pointer(h), ctypes.c_void_p) for h in holders])
        g = tuple(grid) + (1,) * (3 - len(tuple(grid)))
        b = tuple(block) + (1,) * (3 - len(tuple(block)))
        _native.call("sf_launch_kernel", self.function(name), *[int(v) for v in g], *[int(v) for v in b], int(smem),
                     ctypes.c_void_p(stream), argv)

    def bind(self, name: str, grid, block, args: Sequence[object], smem: int = 0, stream: int = 0):
        """A zero-argument callable enqueueing this launch: the argument array is marshalled once,
        so a call costs one C call (timing loops of short kernels stay device-bound)."""
        holders = [a if isinstance(a, ctypes._SimpleCData) else ctypes.c_void_p(int(a)) for a in args]
        argv = (ctypes.c_void_p * len(holders))(*[ctypes.cast(ctypes.pointer(h), ctypes.c_void_p) for h in holders])
        g = [int(v) for v in tuple(grid) + (1,) * (3 - len(tuple(grid)))]
        b = [int(v) for v in tuple(block) + (1,) * (3 - len(tuple(block)))]
        fn, lib = self.function(name), _native.load()
        err = ctypes.create_string_buffer(_native.ERR_CAP)
        st = ctypes.c_void_p(stream)

        def launch() -> None:
            rc = lib.sf_launch_kernel(fn, *g, *b, int(smem), st, argv, err, _native.ERR_CAP)
            if rc != _native.SF_OK:
                raise _native.SfError(rc, err.value.decode(errors="replace"))

        launch.keep = (holders, argv, self)  # the marshalled arguments live as long as the callable
        return launch

    def close(self) -> None:
        if self.handle:
            _native.call("sf_module_unload", self.handle)
            self.handle = None

    def __del__(self):  # best effort: a module outlives no process
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass
