"""The roofline's denominators on this B200: ``calibrate`` (call stack of ``tcenv.cli calibrate``).

Restates tcenv/backends/metal/profile.py: ``measure_peak_bandwidth`` (:73; a 16-byte copy kernel
and a 16-byte read kernel over 512 MiB buffers, two warm-up launches, then the best of five timed
batches of ``iters`` launches), ``measure_peak_flops`` (:123; the vendor GEMM, here cuBLAS through
torch, fp16 and bf16 at n = 4096) and ``effective_peak_gbps`` (:233; the achievable bandwidth
interpolated between the read and the copy figure by the write fraction of a task's minimal
traffic — a pure read stream reaches the read figure, a half-write stream or more the copy
figure).

The probes are this backend's own candidates (compiled and launched through
:mod:`shapeforge_b200.candidates`): every index is bounds-checked against the element count, the
read kernel writes only when its checksum equals a sentinel (so the loads are not removed and
nothing is written in practice).  The result is cached as JSON at ``$SF_CALIBRATION`` or
``~/.cache/shapeforge_b200/calibration-<target>.json`` (the reference caches per target and lets
``TCENV_CALIBRATION`` override, tcenv/target.py:194-204); ``CudaBackend.calibration`` prefers the
pool's measured peaks, then this cache, then the target's shipped ``calibration.json``.
"""

from __future__ import annotations

import json
import os
from pathlib import Path
from typing import Any, Mapping

PROBE_SOURCE = r'''
#include <cstdint>
extern "C" __global__ void copy4(const uint4* __restrict__ x, uint4* __restrict__ y, long long n4) {
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long stride = (long long)gridDim.x * blockDim.x;
    for (; i < n4; i += stride) y[i] = x[i];
}
extern "C" __global__ void read4(const uint4* __restrict__ x, unsigned int* __restrict__ sink, long long n4) {
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    long long stride = (long long)gridDim.x * blockDim.x;
    unsigned int acc = 0;
    for (; i < n4; i += stride) { uint4 v = x[i]; acc ^= v.x ^ v.y ^ v.z ^ v.w; }
    if (acc == 0x9E3779B9u) sink[blockIdx.x] = acc;
}
'''
THREADS = 256
BLOCKS_PER_SM = 8


def cache_file(target_id: str = "b200") -> Path:
    env = os.environ.get("SF_CALIBRATION")
    return Path(env) if env else Path.home() / ".cache" / "shapeforge_b200" / f"calibration-{target_id}.json"


def effective_peak_gbps(read_bytes: float, write_bytes: float, calib: Mapping[str, Any]) -> float:
    """Achievable bandwidth for a read/write mix (profile.py:233-248 interpolation)."""
    wf = float(write_bytes) / max(float(read_bytes) + float(write_bytes), 1.0)
    copy = float(calib.get("copy_gbs") or calib.get("copy_gbps") or calib["peak_gbps"])
    read = float(calib.get("read_gbs") or calib.get("read_gbps") or copy)
    return read - (read - copy) * min(wf / 0.5, 1.0)


def measure_peak_bandwidth(nbytes: int = 512 * 2**20, iters: int = 20) -> dict[str, float]:
    """Best GB/s of the copy (2 bytes moved per byte) and read probes."""
    import ctypes

    import torch

    from .candidates import Module, compile_source

    if nbytes % 16:
        raise ValueError("nbytes must be a multiple of 16")
    mod = Module(compile_source(PROBE_SOURCE, name="calibrate"))
    x = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    y = torch.empty_like(x)
    n4 = nbytes // 16
    sms = torch.cuda.get_device_properties(x.device).multi_processor_count
    grid = (min(-(-n4 // THREADS), sms * BLOCKS_PER_SM), 1, 1)
    sink = torch.zeros(grid[0], dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    args = {
        "copy4": [ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), ctypes.c_longlong(n4)],
        "read4": [ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(sink.data_ptr()), ctypes.c_longlong(n4)],
    }
    out = {}
    for name, moved in (("copy4", 2 * nbytes), ("read4", nbytes)):
        launch = mod.bind(name, grid, (THREADS, 1, 1), args[name], stream=stream)
        for _ in range(2):
            launch()
        torch.cuda.synchronize()
        best = 0.0
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                launch()
            e1.record()
            e1.synchronize()
            per = e0.elapsed_time(e1) / 1e3 / iters
            best = max(best, moved / per / 1e9)
        out[name + "_gbps"] = best
    return out


def measure_peak_flops(n: int = 4096, iters: int = 20) -> dict[str, float]:
    """Best TFLOP/s of the vendor GEMM (cuBLAS through torch) per 16-bit dtype."""
    import torch

    out = {}
    for name, dt in (("fp16", torch.float16), ("bf16", torch.bfloat16)):
        a = torch.randn(n, n, device="cuda", dtype=dt)
        b = torch.randn(n, n, device="cuda", dtype=dt)
        for _ in range(3):
            torch.matmul(a, b)
        torch.cuda.synchronize()
        best = 0.0
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(iters):
                torch.matmul(a, b)
            e1.record()
            e1.synchronize()
            best = max(best, 2.0 * n ** 3 * iters / (e0.elapsed_time(e1) / 1e3) / 1e12)
        out[name] = best
    return out


def calibrate(target_id: str = "b200", *, write: bool = True) -> dict[str, Any]:
    """Measure both peaks on the current device and (by default) cache them."""
    import torch

    from .gpulock import gpu_lock

    with gpu_lock("calibration"):
        bw = measure_peak_bandwidth()
        fl = measure_peak_flops()
    doc = {
        "device": torch.cuda.get_device_name(),
        "copy_gbs": bw["copy4_gbps"],
        "read_gbs": bw["read4_gbps"],
        "peak_tflops": fl,
        "source": "calibrate: 16-byte copy/read probes over 512 MiB (best of 5 x 20); cuBLAS GEMM n=4096",
    }
    if write:
        path = cache_file(target_id)
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(json.dumps(doc, indent=1, sort_keys=True) + "\n")
    return doc


if __name__ == "__main__":
    print(json.dumps(calibrate(), indent=1, sort_keys=True))
