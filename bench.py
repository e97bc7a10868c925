"""Benchmark of the ShapeForge B200 backend's hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A *step* is one evaluation of the workload's shard: one launch of the task operator over one
set of synthetic inputs resident in HBM.  Inputs rotate over several sets whose total size is
larger than the 126 MB L2, so every timed launch reads its operands from HBM (the reference's
``fresh_rotation`` discipline, tcenv/track/protocol.py:230).  Timing: W untimed warm-up steps,
then exactly K steps between a barrier + synchronize on both sides, CUDA events on the
launching stream, max over ranks.

The default workload is the dense-gemm configuration: C = A . B^T with A, B fp16
[4096, 4096] ~ U(-1, 1), fp32 accumulation, fp16 output.  Other workloads (``--workload``)
cover the remaining task operators for per-shard reports.

``--impl reference`` times the reference's CPU algorithm for the same workload (the oracle
port in ``oracle/``, which restates the task's ``reference.py``) on the host cores; under
torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Callable

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "per-shard latency and % roofline (HBM GB/s or TC TFLOPS) per OpSpec task"
# Forced kernel variant of the operator workloads (--variant; 0 = the default dispatch).
VARIANT = 0
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def measured_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            return json.loads(p.read_text()), "measured"
        except (OSError, ValueError):
            pass
    return dict(FALLBACK_PEAKS), "fallback"


# ---- clocks ---------------------------------------------------------------------------------


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML in a background thread."""

    REASONS = {
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
        0x0000000000000004: "sw_power_cap",
        0x0000000000000002: "applications_clocks_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.period = period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = int(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception:  # NVML absent (CPU box): no clock record
            self._nvml = None

    def _sample(self):
        nv = self._nvml
        try:
            mhz = int(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
            reasons = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            self.samples.append((mhz, reasons))
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            self._stop.wait(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._sample()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
            self._sample()

    def summary(self) -> dict | None:
        if self._nvml is None or not self.samples:
            return None
        mhz = [s[0] for s in self.samples]
        seen = 0
        for _, r in self.samples:
            seen |= r
        reasons = sorted(name for bit, name in self.REASONS.items() if seen & bit)
        return {"sm_mhz": float(statistics.median(mhz)), "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(mhz)}


# ---- workloads ------------------------------------------------------------------------------


@dataclass
class Workload:
    name: str
    unit: str  # "TFLOP/s" or "GB/s"
    bound: str  # "tensor" or "hbm"
    dtype: str
    units_per_step: float  # algorithmic flops or bytes of one launch
    config: dict
    kernel: str  # dominant kernel name (ncu)
    make_sets: Callable  # (device, nsets) -> list of (tensors tuple, pointer list)
    desc: Callable  # () -> sf_op_desc
    host_inputs: Callable  # () -> (list of pinned host input tensors, list of output shapes/dtypes)
    e2e_launch: Callable  # (device inputs, device outputs, stream) -> None: the public C-ABI call
    cpu_rows: Callable  # (rows) -> (callable running the oracle on a row sample, units of that call, description)
    total_rows: int  # rows of the full shard (the sample is a row subset; rows are independent)
    nsets: int = 4
    launches_per_step: int = 1
    # Head-sharded workloads (attention, KDA): this rank's share of the job and the whole job's
    # units per step; replicated workloads leave these at their defaults.
    sharded: bool = False
    total_units: float | None = None
    shard_note: str = ""
    # CPU tensors of the workload at the search seed (for the registered-baseline timing).
    cpu_inputs: Callable | None = None
    # Steps of several launches: what `achieved` and `traffic` cover.
    roofline_note: str = ""


def _gemm_nt_workload(m: int, n: int, k: int, dtype: str = "fp16") -> Workload:
    import numpy as np
    import torch

    from shapeforge_b200 import _native, cases

    td = cases.TORCH_DTYPE[dtype]
    per_set = 2 * (m * k + n * k + m * n)
    nsets = max(2, int(np.ceil(2 * L2_BYTES / per_set)))
    flops = 2.0 * m * n * k

    def make_sets(dev, count):
        out = []
        for s in range(count):
            inp = cases.gemm_bench_inputs(m, n, k, dtype, seed=cases.SEARCH_SEED + s)
            a, b = inp["A"].to(dev), inp["B"].to(dev)
            c = torch.empty((m, n), dtype=td, device=dev)
            out.append(((a, b, c), [a.data_ptr(), b.data_ptr(), c.data_ptr()]))
        return out

    def desc():
        return _native.op_desc("gemm_nt", dtype, dims=(m, n, k))

    def host_inputs():
        inp = cases.gemm_bench_inputs(m, n, k, dtype, seed=cases.SEARCH_SEED)
        return [inp["A"].pin_memory(), inp["B"].pin_memory()], [((m, n), td)]

    def e2e_launch(d_in, d_out, stream):
        _native.call("sf_gemm_nt", d_in[0].data_ptr(), d_in[1].data_ptr(), d_out[0].data_ptr(), m, n, k,
                     _native.DTYPE_CODES[dtype], stream)

    def cpu_rows(rows):
        # The reference's algorithm (tasks/gemm/reference.py:110-114: an fp32 product) through
        # the oracle port, on a row sample of the same workload (output rows are independent).
        from oracle import ops as oref

        inp = cases.gemm_bench_inputs(rows, n, k, dtype, seed=cases.SEARCH_SEED)
        a = inp["A"].float().numpy()
        b = inp["B"].float().numpy()
        return (lambda: oref.gemm_nt(a, b)), 2.0 * rows * n * k, f"fp32 A[{rows},{k}] . B[{n},{k}]^T (row sample)"

    return Workload(
        name=f"gemm_nt_{m}x{n}x{k}",
        unit="TFLOP/s",
        bound="tensor",
        dtype=dtype,
        units_per_step=flops,
        config={
            "workload": f"dense gemm C=A.B^T, A {dtype} [{m},{k}], B {dtype} [{n},{k}], fp32 accumulate, {dtype} out",
            "shape": [m, n, k],
            "inputs": "U(-1,1), seed 7",
            "l2": f"inputs rotate over {nsets} sets ({nsets * per_set / 2**20:.0f} MiB) > L2 126 MB",
        },
        # One 128 x 64 tile per SM or fewer: the small-problem kernel (B200: 148 SMs).
        kernel="gemm_nt_small_kernel" if -(-m // 128) * -(-n // 64) <= 148 else "gemm_nt_tc_kernel",
        make_sets=make_sets,
        desc=desc,
        host_inputs=host_inputs,
        e2e_launch=e2e_launch,
        cpu_rows=cpu_rows,
        total_rows=m,
        nsets=nsets,
        cpu_inputs=lambda: cases.gemm_bench_inputs(m, n, k, dtype, seed=cases.SEARCH_SEED),
    )


def _rmsnorm_workload(rows: int, hidden: int, dtype: str = "fp16") -> Workload:
    import numpy as np
    import torch

    from shapeforge_b200 import _native, cases

    td = cases.TORCH_DTYPE[dtype]
    nbytes = 4.0 * rows * hidden + 2.0 * hidden
    per_set = nbytes
    nsets = max(2, int(np.ceil(2 * L2_BYTES / per_set)))

    def make_sets(dev, count):
        out = []
        for s in range(count):
            inp = cases.rmsnorm_bench_inputs(rows, hidden, dtype, seed=cases.SEARCH_SEED + s)
            x, w = inp["x"].to(dev), inp["w"].to(dev)
            y = torch.empty_like(x)
            out.append(((x, w, y), [x.data_ptr(), w.data_ptr(), y.data_ptr()]))
        return out

    def desc():
        return _native.op_desc("rmsnorm", dtype, dims=(rows, hidden), attrs=(1e-6,))

    def host_inputs():
        inp = cases.rmsnorm_bench_inputs(rows, hidden, dtype)
        return [inp["x"].pin_memory(), inp["w"].pin_memory()], [((rows, hidden), td)]

    def e2e_launch(d_in, d_out, stream):
        _native.call("sf_rmsnorm", d_in[0].data_ptr(), d_in[1].data_ptr(), d_out[0].data_ptr(), rows, hidden, 1e-6,
                     _native.DTYPE_CODES[dtype], stream)

    def cpu_rows(r):
        from oracle import ops as oref

        inp = cases.rmsnorm_bench_inputs(r, hidden, dtype)
        x = inp["x"].double().numpy()
        w = inp["w"].double().numpy()
        return (lambda: oref.rmsnorm(x, w, 1e-6)), 4.0 * r * hidden + 2.0 * hidden, f"fp64 oracle on [{r},{hidden}] (row sample)"

    return Workload(
        name=f"rmsnorm_{rows}x{hidden}",
        unit="GB/s",
        bound="hbm",
        dtype=dtype,
        units_per_step=nbytes,
        config={
            "workload": f"rmsnorm x {dtype} [{rows},{hidden}] ~ N(0,1), w U(0.5,1.5), eps 1e-6, fp32 accumulate",
            "shape": [rows, hidden],
            "l2": f"inputs rotate over {nsets} sets ({nsets * per_set / 2**20:.0f} MiB) > L2 126 MB",
        },
        kernel="rmsnorm_warp_kernel" if hidden <= 1024 else "rmsnorm_vec_kernel",  # a warp per row up to 1024 elements
        make_sets=make_sets,
        desc=desc,
        host_inputs=host_inputs,
        e2e_launch=e2e_launch,
        cpu_rows=cpu_rows,
        total_rows=rows,
        nsets=nsets,
        cpu_inputs=lambda: cases.rmsnorm_bench_inputs(rows, hidden, dtype),
    )


def _op_workload(name, unit, bound, dtype, units, config, kernel, op, make_inputs, in_names, out_specs, dims, attrs=(), flags=0,
                 cpu_rows=None, total_rows=1, null_args=(), scratch_bytes=0, launches_per_step=1, roofline_note="") -> Workload:
    """A workload over one C-ABI operator: ``make_inputs(seed)`` gives CPU tensors named
    ``in_names`` (ABI order, followed by the outputs ``out_specs`` = [(shape, dtype)]);
    ``null_args`` are ABI positions passed as NULL (optional tensors); ``scratch_bytes`` > 0
    appends a device workspace of that size (one per device, launches are stream-ordered)."""
    import numpy as np
    import torch

    from shapeforge_b200 import _native

    sample = make_inputs(cases_seed())
    per_set = sum(t.numel() * t.element_size() for t in sample.values()) + sum(
        int(np.prod(s)) * torch.tensor([], dtype=dt).element_size() for s, dt in out_specs)
    nsets = max(2, int(np.ceil(2 * L2_BYTES / per_set)))
    scratch = {}

    def scratch_ptr(dev):
        if not scratch_bytes:
            return []
        if dev not in scratch:
            scratch[dev] = torch.empty(scratch_bytes, dtype=torch.uint8, device=dev)
        return [scratch[dev].data_ptr()]

    def ptr_list(ins, outs, dev):
        ptrs = [ins[n].data_ptr() for n in in_names] + [o.data_ptr() for o in outs]
        for pos in null_args:
            ptrs.insert(pos, 0)
        return ptrs + scratch_ptr(dev)

    def make_sets(dev, count):
        out = []
        for s in range(count):
            ins = {k: v.to(dev) for k, v in make_inputs(cases_seed() + s).items()}
            outs = [torch.empty(shape, dtype=dt, device=dev) for shape, dt in out_specs]
            out.append(((ins, outs), ptr_list(ins, outs, dev)))
        return out

    def desc():
        return _native.op_desc(op, dtype, dims=dims, attrs=attrs, flags=flags, variant=VARIANT)

    def host_inputs():
        ins = make_inputs(cases_seed())
        return [ins[n].pin_memory() for n in in_names], list(out_specs)

    def e2e_launch(d_in, d_out, stream):
        ptrs = [t.data_ptr() for t in d_in] + [o.data_ptr() for o in d_out]
        for pos in null_args:
            ptrs.insert(pos, 0)
        _native.run_op(desc(), ptrs + scratch_ptr(d_in[0].device), stream)

    return Workload(name=name, unit=unit, bound=bound, dtype=dtype, units_per_step=units,
                    config=dict(config, l2=f"inputs rotate over {nsets} sets ({nsets * per_set / 2**20:.0f} MiB) > L2 126 MB"),
                    kernel=kernel, make_sets=make_sets, desc=desc, host_inputs=host_inputs, e2e_launch=e2e_launch,
                    cpu_rows=cpu_rows, total_rows=total_rows, nsets=nsets, launches_per_step=launches_per_step,
                    roofline_note=roofline_note,
                    cpu_inputs=lambda: make_inputs(cases_seed()))


def cases_seed() -> int:
    from shapeforge_b200 import cases

    return cases.SEARCH_SEED


def _attention_workload(b: int, h: int, s: int, d: int, causal: bool = True, dtype: str = "bf16", world: int = 1,
                        rank: int = 0) -> Workload:
    """With world > 1 the b*h heads are split into contiguous ranges, one per rank (each rank's
    slice is a [1, n_r, s, d] problem); the job's units are the full problem's flops."""
    import math

    import torch

    from shapeforge_b200 import cases, shard

    scale = 1.0 / math.sqrt(d)
    total_flops = 4.0 * b * h * d * (s * (s + 1) / 2 if causal else s * s)
    full_shape = (b, h, s, d)
    if world > 1:
        h0, h1 = shard.head_ranges(b * h, world)[rank]
        shape = (1, h1 - h0, s, d)
    else:
        shape = full_shape
    flops = total_flops * (shape[0] * shape[1]) / (b * h)

    def make_inputs(seed):
        return cases.attention_bench_inputs(shape, dtype, seed=seed + 1000 * rank)

    def cpu_rows(rows):
        # The reference's algorithm (tasks/flash_attention/reference.py:113-119 with the causal
        # mask) through the oracle port, on the last `rows` query rows of one head.
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        q = inp["q"][:1, :1].float().numpy()
        k = inp["k"][:1, :1].float().numpy()
        v = inp["v"][:1, :1].float().numpy()
        sel = list(range(s - rows, s))
        fl = sum(4.0 * d * ((i + 1) if causal else s) for i in sel)
        return (lambda: oref.attention_rows(q, k, v, scale, causal, sel)), fl, f"fp64 attention of {rows} query rows x one head"

    wl = _op_workload(
        f"attention_{'causal' if causal else 'full'}_{b}x{h}x{s}x{d}", "TFLOP/s", "tensor", dtype, flops,
        {"workload": f"flash attention forward {'causal' if causal else 'non-causal'}, q/k/v {dtype} [{b},{h},{s},{d}] ~ N(0,1), "
                     f"scale 1/sqrt({d}), fp32 softmax statistics", "shape": [b, h, s, d]},
        # At most one (b*h, 128-row query tile) CTA per SM (B200: 148): the S-double-buffered kernel.
        "fa_fwd_db_kernel" if shape[0] * shape[1] * -(-s // 128) <= 148 else "fa_fwd_kernel",
        "flash_attention", make_inputs, ["q", "k", "v"], [(shape, cases.TORCH_DTYPE[dtype])],
        shape, (scale,), 1 if causal else 0, cpu_rows=cpu_rows, total_rows=s)
    if world > 1:
        wl.sharded, wl.total_units = True, total_flops
        wl.shard_note = f"b*h={b * h} heads split into {world} contiguous ranges (rank {rank}: {shape[1]} heads)"
    return wl


def _bitdelta_base_workload(m: int, n: int = 4096, k: int = 4096, dtype: str = "fp16") -> Workload:
    import torch

    from shapeforge_b200 import cases

    nbytes = 2.0 * n * k + n * k / 8 + 2.0 * n + 2.0 * m * k + 2.0 * m * n

    def make_inputs(seed):
        return cases.bitdelta_base_inputs("normal", seed, m, n, k, dtype)

    def cpu_rows(rows):
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        x = inp["x"][:1].double().numpy()
        w = inp["w_base"][:rows].double().numpy()
        sw = inp["s_words"][:rows].numpy()
        a = inp["alpha"][:rows].double().numpy()
        fb = 2.0 * rows * k + rows * k / 8 + 2.0 * rows
        return (lambda: oref.bitdelta_gemm_base(x, w, sw, a)), fb, f"fp64 oracle over {rows} output columns (W_base rows)"

    return _op_workload(
        f"bitdelta_base_m{m}", "GB/s", "hbm", dtype, nbytes,
        {"workload": f"bitdelta y = x.(W_base + diag(alpha) S)^T, x {dtype} [{m},{k}] ~ N(0,1), W_base {dtype} [{n},{k}] ~ N(0,0.02), "
                     f"S Bernoulli(0.5) packed u32 [{n},{k // 32}], alpha {dtype} U(1e-3,1e-2)", "shape": [m, n, k]},
        "bitdelta_base_stream_kernel" if m <= 4 else "bitdelta_base_kernel", "bitdelta_gemm_base", make_inputs, ["x", "w_base", "s_words", "alpha"],
        [((m, n), cases.TORCH_DTYPE[dtype])], (m, n, k), cpu_rows=cpu_rows, total_rows=n)


# The two-pass KDA step is three launches (chunk prefix, parallel chunk preparation, state chains).
KDA_ROOFLINE_NOTE = ("step of 3 launches (kda_slots_kernel, kda_prep_kernel, kda_chain_kernel): achieved = algorithmic bytes "
                     "/ step time; traffic = the named (longest) kernel's DRAM bytes per launch")


def _kda_gated_workload(heads: int = 16, dim: int = 128, dtype: str = "bf16", world: int = 1, rank: int = 0) -> Workload:
    """With world > 1 the 8 x H (sequence, head) chains are dealt to ranks by a token balance
    (``shard.chain_assign``) and each rank runs its chains repacked as a single-head packed batch;
    the job's units are the full problem's bytes."""
    import math

    import torch

    from shapeforge_b200 import cases, ops, shard

    lengths = cases.kda_gated_lengths()
    total = int(sum(lengths))
    n = len(lengths)
    per_token = 3 * 2 * dim + 4 * dim + 4 + 2 * dim  # q, k, v, g, beta in; out
    total_bytes = per_token * heads * total + 4.0 * n * heads * dim * dim
    cu = [0]
    for x in lengths:
        cu.append(cu[-1] + x)
    chains = shard.chain_assign(lengths, heads, world)[rank] if world > 1 else None

    if chains is None:
        def make_inputs(seed):
            return cases.kda_gated_inputs(lengths, heads, dim, dtype, seed=seed)

        ws = ops.varlen_kda_gated_workspace_bytes(total, n, heads, dim)
        dims, out_specs = (n, heads, dim, total, ws), [((total, heads, dim), cases.TORCH_DTYPE[dtype]), ((n, heads, dim, dim), torch.float32)]
        nbytes = total_bytes
    else:
        cu_r = shard.chain_offsets(cu, chains)
        t_r = cu_r[-1]

        def make_inputs(seed):
            full = cases.kda_gated_inputs(lengths, heads, dim, dtype, seed=seed)
            packed = {k: shard.pack_chains(full[k], cu, chains) for k in ("q", "k", "v", "g", "beta")}
            packed["cu_seqlens"] = torch.tensor(cu_r, dtype=torch.int32)
            return packed

        ws = ops.varlen_kda_gated_workspace_bytes(t_r, len(chains), 1, dim)
        dims, out_specs = (len(chains), 1, dim, t_r, ws), [((t_r, 1, dim), cases.TORCH_DTYPE[dtype]), ((len(chains), 1, dim, dim), torch.float32)]
        nbytes = per_token * t_r + 4.0 * len(chains) * dim * dim

    def cpu_rows(rows):
        # The delta-rule recurrence (tasks/varlen_kda/reference.py:352-368, gate supplied) through
        # the oracle port on the first `rows` tokens of one (sequence, head) chain.
        from oracle import ops as oref

        inp = cases.kda_gated_inputs(lengths, 1, dim, dtype, seed=cases.SEARCH_SEED)
        t = min(rows, lengths[0])
        f = lambda name: inp[name][:t, :1].double().numpy()  # noqa: E731
        return ((lambda: oref.varlen_kda_gated(f("q"), f("k"), f("v"), f("g"), f("beta"), [0, t], 1.0 / math.sqrt(dim))),
                per_token * float(t), f"fp64 recurrence over {t} tokens of one chain")

    wl = _op_workload(
        "kda_gated", "GB/s", "hbm", dtype, nbytes,
        {"workload": f"varlen gated KDA, {n} packed sequences {lengths} (seeded U(256,4096)), H={heads}, D={dim}, q/k {dtype} "
                     "L2-normalised, v {dtype}, beta=sigmoid(N) fp32, g=logsigmoid(N) fp32, zero initial state".replace("{dtype}", dtype),
         "total_tokens": total},
        "kda_prep_kernel", "varlen_kda_gated", make_inputs, ["q", "k", "v", "g", "beta", "cu_seqlens"], out_specs, dims,
        (1.0 / math.sqrt(dim),), cpu_rows=cpu_rows, total_rows=lengths[0], null_args=(6,), scratch_bytes=ws, launches_per_step=3)
    wl.roofline_note = KDA_ROOFLINE_NOTE
    if chains is not None:
        wl.sharded, wl.total_units = True, total_bytes
        wl.shard_note = (f"{n}x{heads} (sequence, head) chains dealt to {world} ranks by token count (rank {rank}: "
                         f"{len(chains)} chains, {t_r} token-heads), repacked as single-head batches")
    return wl


def _mamba2_workload(b: int = 2, l: int = 2048, h: int = 8, p: int = 64, n: int = 64, c: int = 64, dtype: str = "fp16") -> Workload:
    """The mamba2_chunk_scan paper size (tasks/mamba2_chunk_scan/opspec.json sizes.paper)."""
    from shapeforge_b200 import cases

    nc = l // c

    def nbytes(bb, chunks):
        rows = bb * chunks * c
        return 2.0 * (2 * rows * h * p + 2 * rows * h + 2 * rows * n + h + bb * chunks * h * p * n)

    def make_inputs(seed):
        return cases.mamba2_inputs("normal", seed, b, l, h, p, n, c, dtype)

    def cpu_rows(rows):
        # tasks/mamba2_chunk_scan/reference.py:106-127 through the oracle port, on the first `rows`
        # chunks of batch 0 (chunks are independent).
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        k = min(rows, nc)
        t = k * c
        a = [inp["x"][:1, :t], inp["dt"][:1, :t], inp["dA_cumsum"][:1, :, :k], inp["Bmat"][:1, :t], inp["Cmat"][:1, :t],
             inp["Dskip"], inp["states"][:1, :k]]
        a = [v.double().numpy() for v in a]
        return (lambda: oref.mamba2_chunk_scan(*a)), nbytes(1, k), f"fp64 oracle over {k} chunks of batch 0"

    return _op_workload(
        f"mamba2_chunk_scan_b{b}_l{l}_h{h}", "GB/s", "hbm", dtype, nbytes(b, nc),
        {"workload": f"mamba2 SSD chunk scan, B={b} L={l} H={h} P={p} N={n} CHUNK={c}, {dtype}, task input stream "
                     "(normal case: x/B/C/D/states ~ N(0,1), dt in [0.001,0.05], A in [-8,-1])", "shape": [b, l, h, p, n, c]},
        "mamba2_tc_kernel", "mamba2_chunk_scan", make_inputs, ["x", "dt", "dA_cumsum", "Bmat", "Cmat", "Dskip", "states"],
        [((b, l, h, p), cases.TORCH_DTYPE[dtype])], (b, l, h, p, n, c), cpu_rows=cpu_rows, total_rows=nc)


def _membound_task_workload(task: str, shape, dtype: str = "fp16", kernel: str = "") -> Workload:
    """A memory-bound task at its reference paper size (tasks/<task>/opspec.json sizes.paper),
    inputs from the task's own stream (normal case); units = the opspec's min_bytes (inputs and
    outputs, each once)."""
    import math

    import numpy as np

    from shapeforge_b200 import cases

    el = 2
    n_elem = int(np.prod(shape))
    if task == "reduction_sum":
        m, n = shape
        nbytes, outs, dims = el * m * n + el * m, [((m,), cases.TORCH_DTYPE[dtype])], (m, n)
    elif task == "swiglu":
        nbytes, outs, dims = 3 * el * n_elem, [(tuple(shape), cases.TORCH_DTYPE[dtype])], (n_elem,)
    elif task == "rope":
        nbytes, outs, dims = 2 * el * n_elem, [(tuple(shape), cases.TORCH_DTYPE[dtype])], tuple(shape)
    elif task in ("silu", "relu", "sigmoid", "sigmoid_shift"):
        nbytes, outs, dims = 2 * el * n_elem, [(tuple(shape), cases.TORCH_DTYPE[dtype])], (n_elem,)
    else:  # softmax
        m, n = shape
        nbytes, outs, dims = 2 * el * m * n, [(tuple(shape), cases.TORCH_DTYPE[dtype])], (m, n)
    names = ["gate", "up"] if task == "swiglu" else ["x"]
    attrs = (10000.0,) if task == "rope" else ()
    block = shape[-1] if task in ("softmax", "reduction_sum") else (shape[-2] * shape[-1] if task == "rope" else 65536)
    total_rows = max(1, n_elem // block)

    def make_inputs(seed):
        return cases.membound_inputs(task, "normal", seed, shape, dtype)

    def cpu_rows(rows):
        # The task's reference formula through the oracle port on the first `rows` rows (blocks).
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        k = rows * block
        if task == "swiglu":
            g = inp["gate"].reshape(-1)[:k].double().numpy()
            u = inp["up"].reshape(-1)[:k].double().numpy()
            return (lambda: oref.swiglu(g, u)), 3.0 * el * k, f"fp64 swiglu of {k} elements"
        x = inp["x"].reshape(-1)[:k].double().numpy()
        if task == "rope":
            xr = x.reshape(rows, shape[-2], shape[-1])
            return (lambda: oref.rope(xr, 10000.0)), 2.0 * el * k, f"fp64 rope of {rows} heads"
        if task in ("softmax", "reduction_sum"):
            xr = x.reshape(rows, shape[-1])
            fn = oref.softmax if task == "softmax" else oref.reduction_sum
            per = (2 * el * k) if task == "softmax" else (el * k + el * rows)
            return (lambda: fn(xr)), float(per), f"fp64 {task} of {rows} rows"
        fn = {"silu": oref.silu, "relu": oref.relu, "sigmoid": oref.sigmoid, "sigmoid_shift": oref.sigmoid_shift}[task]
        return (lambda: fn(x)), 2.0 * el * k, f"fp64 {task} of {k} elements"

    label = "x".join(str(v) for v in shape)
    return _op_workload(
        f"{task}_{label}", "GB/s", "hbm", dtype, nbytes,
        {"workload": f"task {task} at the reference paper size {list(shape)}, {dtype}, the task's normal-case input stream",
         "shape": list(shape)},
        kernel, task, make_inputs, names, outs, dims, attrs, cpu_rows=cpu_rows, total_rows=total_rows)


def _gemm_nn_task_workload(m: int = 2048, n: int = 2048, k: int = 2048, dtype: str = "fp16") -> Workload:
    """tasks/gemm (C = A.B, B stored [K, N]) at its paper size; the tensor-core kernel reads B in
    place as an MN-major operand (the workspace argument of the C ABI is passed but not needed)."""
    import torch

    from shapeforge_b200 import cases

    ws = 2 * n * k

    def make_inputs(seed):
        return cases.gemm_inputs("normal", seed, (m, k), (k, n), dtype)

    def cpu_rows(rows):
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        a = inp["A"][:rows].float().numpy()
        b = inp["B"].float().numpy()
        return (lambda: a @ b), 2.0 * rows * n * k, f"fp32 A[{rows} rows,{k}] . B[{k},{n}] (row sample)"

    wl = _op_workload(
        f"gemm_nn_{m}x{n}x{k}", "TFLOP/s", "tensor", dtype, 2.0 * m * n * k,
        {"workload": f"task gemm C=A.B, A {dtype} [{m},{k}], B {dtype} [{k},{n}] (K x N, read in place as an MN-major operand), "
                     "fp32 accumulate", "shape": [m, n, k]},
        "gemm_nt_tc_kernel", "gemm_nn", make_inputs, ["A", "B"], [((m, n), cases.TORCH_DTYPE[dtype]), ((ws,), torch.uint8)],
        (m, n, k, ws), cpu_rows=cpu_rows, total_rows=m)
    return wl


def _lion_task_workload(n: int = 8388608, dtype: str = "fp16") -> Workload:
    """tasks/lion at its paper size: one optimizer step over N parameters (p, g, m in; p_out, m_out
    out); units = the opspec's min_bytes, 5 tensors of N 16-bit elements."""
    from shapeforge_b200 import cases

    el = 2
    a = cases.LION_DEFAULTS

    def make_inputs(seed):
        return cases.lion_inputs("normal", seed, n, dtype)

    def cpu_rows(rows):
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        k = rows * 65536
        p, g, m = (inp[name][:k].double().numpy() for name in ("p", "g", "m"))
        return (lambda: oref.lion(p, g, m, a["LR"], a["WD"], a["BETA1"], a["BETA2"])), 5.0 * el * k, f"fp64 lion step of {k} elements"

    td = cases.TORCH_DTYPE[dtype]
    return _op_workload(
        f"lion_{n}", "GB/s", "hbm", dtype, 5.0 * el * n,
        {"workload": f"task lion (one Lion step, LR/WD/BETA1/BETA2 = opspec defaults) over N={n} {dtype} parameters, "
                     "the task's normal-case input stream", "shape": [n]},
        "lion_kernel", "lion", make_inputs, ["p", "g", "m"], [((n,), td), ((n,), td)], (n,),
        (a["LR"], a["WD"], a["BETA1"], a["BETA2"]), cpu_rows=cpu_rows, total_rows=max(1, n // 65536))


def _gemv_task_workload(m: int = 4096, k: int = 4096, dtype: str = "fp16") -> Workload:
    """tasks/gemv at its paper size; units = the opspec's min_bytes (A, x, y once)."""
    from shapeforge_b200 import cases

    el = 2

    def make_inputs(seed):
        return cases.gemv_inputs("normal", seed, m, k, dtype)

    def cpu_rows(rows):
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        a_np = inp["A"][:rows].double().numpy()
        x_np = inp["x"].double().numpy()
        return (lambda: oref.gemv(a_np, x_np)), float(el * (rows * k + k + rows)), f"fp64 gemv of {rows} rows x K={k}"

    return _op_workload(
        f"gemv_{m}x{k}", "GB/s", "hbm", dtype, float(el * (m * k + k + m)),
        {"workload": f"task gemv y = A.x, A {dtype} [{m},{k}], the task's normal-case input stream", "shape": [m, k]},
        "gemv_kernel", "gemv", make_inputs, ["A", "x"], [((m,), cases.TORCH_DTYPE[dtype])], (m, k),
        cpu_rows=cpu_rows, total_rows=m)


def _gemm_silu_task_workload(m: int = 2048, n: int = 2048, k: int = 2048, dtype: str = "fp16") -> Workload:
    """tasks/gemm_silu (C = silu(A.B), B stored [K, N]) at its paper size; units = the opspec's
    flops 2*M*N*K + 5*M*N."""
    import torch

    from shapeforge_b200 import cases

    ws = 2 * n * k

    def make_inputs(seed):
        return cases.gemm_inputs("normal", seed, (m, k), (k, n), dtype)

    def cpu_rows(rows):
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        a = inp["A"][:rows].double().numpy()
        b = inp["B"].double().numpy()
        return (lambda: oref.gemm_silu(a, b)), 2.0 * rows * n * k + 5.0 * rows * n, f"fp64 silu(A[{rows} rows,{k}] . B[{k},{n}])"

    return _op_workload(
        f"gemm_silu_{m}x{n}x{k}", "TFLOP/s", "tensor", dtype, 2.0 * m * n * k + 5.0 * m * n,
        {"workload": f"task gemm_silu C=silu(A.B), A {dtype} [{m},{k}], B {dtype} [{k},{n}] read in place as an MN-major "
                     "operand, SiLU fused into the tensor-core epilogue", "shape": [m, n, k]},
        "gemm_nt_tc_kernel", "gemm_silu", make_inputs, ["A", "B"], [((m, n), cases.TORCH_DTYPE[dtype]), ((ws,), torch.uint8)],
        (m, n, k, ws), cpu_rows=cpu_rows, total_rows=m)


def _kda_fixed_task_workload(n: int = 256, h: int = 8, d: int = 64, dtype: str = "fp16") -> Workload:
    """tasks/kda (fixed length, one sequence) at its paper size; units = the opspec's min_bytes:
    q, k, v, g and output (N*H*D each, 16-bit) plus initial_state and final_state (H*D*D fp32)."""
    import torch

    from shapeforge_b200 import cases

    el = 2
    nbytes = 5.0 * el * n * h * d + 2.0 * 4 * h * d * d
    td = cases.TORCH_DTYPE[dtype]

    def make_inputs(seed):
        return cases.kda_fixed_inputs("normal", seed, n, h, d, dtype)

    def cpu_rows(rows):
        # The oracle on the first `rows` heads (heads are independent chains).
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        f = lambda k: inp[k].double().numpy()  # noqa: E731
        q, k, v, g, b = (f(x)[:, :rows] for x in ("q", "k", "v", "g", "beta"))
        a_log = f("A_log")[:rows]
        dt_bias = f("dt_bias").reshape(h, d)[:rows].reshape(-1)
        s0 = f("initial_state")[:rows]
        sc = float(f("scale")[0])
        units = nbytes * rows / h
        return (lambda: oref.kda_fixed(q, k, v, g, b, a_log, dt_bias, s0, sc, -5.0)), units, f"fp64 kda of {rows} heads x {n} tokens"

    return _op_workload(
        f"kda_fixed_{n}x{h}x{d}", "GB/s", "hbm", dtype, nbytes,
        {"workload": f"task kda (fixed length, one sequence) N={n} H={h} D={d} {dtype}, LOWER_BOUND -5, the task's normal-case "
                     "input stream", "shape": [n, h, d]},
        "kda_fwd_kernel", "kda", make_inputs, ["q", "k", "v", "g", "beta", "A_log", "dt_bias", "initial_state", "scale"],
        [((n, h, d), td), ((h, d, d), torch.float32), ((3, 2), torch.int32), ((1,), torch.int32), ((2, h, d, d), torch.float32)],
        (n, h, d), (-5.0,), cpu_rows=cpu_rows, total_rows=h, launches_per_step=2,
        roofline_note="step of 2 launches (kda_fixed_items_kernel writes the one-piece work list, kda_fwd_kernel runs the "
                      "recurrence): achieved = algorithmic bytes / step time")


def _bitdelta_task_workload(m: int = 512, n: int = 4096, k: int = 4096, dtype: str = "fp16", scale: float = 0.02) -> Workload:
    """tasks/bitdelta_gemm (y = SCALE x.W, W +-1 from bits [K/32, N]) at its paper size."""
    from shapeforge_b200 import cases

    def make_inputs(seed):
        return cases.bitdelta_inputs("random", seed, m, n, k, dtype)

    def cpu_rows(rows):
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        x = inp["x"][:rows].double().numpy()
        bits = inp["bits"].numpy()
        return (lambda: oref.bitdelta_gemm(x, bits, scale)), 2.0 * rows * n * k, f"fp64 oracle over {rows} rows of x"

    return _op_workload(
        f"bitdelta_gemm_{m}x{n}x{k}", "TFLOP/s", "tensor", dtype, 2.0 * m * n * k,
        {"workload": f"task bitdelta_gemm y = {scale} x.W, x {dtype} [{m},{k}] ~ N(0,1), W +-1 from uniform 32-bit words "
                     f"[{k // 32},{n}]", "shape": [m, n, k]},
        "bitdelta_task_kernel", "bitdelta_gemm", make_inputs, ["x", "bits"], [((m, n), cases.TORCH_DTYPE[dtype])], (m, n, k),
        (scale,), cpu_rows=cpu_rows, total_rows=m)


def _kda_task_workload(heads: int = 64, dim: int = 128, lengths=(2048, 1024, 1024, 2048, 1024, 1024), dtype: str = "bf16") -> Workload:
    """tasks/varlen_kda (in-op q/k norms, gates from A_log / dt_bias, sigmoid beta, initial state)
    at the v6_h64_mixed size; units = the opspec's min_bytes (q, k, v, g, output, initial and final
    state)."""
    import math

    import torch

    from shapeforge_b200 import cases

    lengths = list(lengths)
    t = int(sum(lengths))
    n = len(lengths)
    nbytes = 5.0 * 2 * t * heads * dim + 2.0 * 4 * n * heads * dim * dim

    def make_inputs(seed):
        return cases.kda_task_inputs(lengths, heads, dim, dtype, seed)

    def cpu_rows(rows):
        # tasks/varlen_kda/reference.py:323-374 through the oracle port on the first `rows` tokens of
        # one (sequence, head) chain.
        from oracle import ops as oref

        inp = make_inputs(cases.SEARCH_SEED)
        tt = min(rows, lengths[0])
        f = lambda name: inp[name][:tt, :1].double().numpy()  # noqa: E731
        args = (f("q"), f("k"), f("v"), f("g"), inp["beta"][:tt, :1].double().numpy(), inp["A_log"][:1].double().numpy(),
                inp["dt_bias"][:dim].double().numpy(), inp["initial_state"][:1, :1].double().numpy(), [0, tt],
                float(inp["scale"][0]), -5.0)
        return (lambda: oref.varlen_kda(*args)), 5.0 * 2 * tt * dim + 2.0 * 4 * dim * dim, f"fp64 recurrence over {tt} tokens of one chain"

    from shapeforge_b200 import ops

    ws = ops.varlen_kda_workspace_bytes(t, n, heads, dim)
    return _op_workload(
        f"varlen_kda_h{heads}_mixed", "GB/s", "hbm", dtype, nbytes,
        {"workload": f"task varlen_kda v6_h64_mixed: {n} sequences {lengths}, H={heads}, D={dim}, {dtype}, the task's input "
                     "stream (0.5 N(0,1) q/k/v/g/beta, A_log = log U(1,16), dt_bias, non-zero initial state)", "total_tokens": t},
        "kda_prep_kernel", "varlen_kda", make_inputs,
        ["q", "k", "v", "g", "beta", "A_log", "dt_bias", "initial_state", "cu_seqlens", "scale"],
        [((t, heads, dim), cases.TORCH_DTYPE[dtype]), ((n, heads, dim, dim), torch.float32)], (n, heads, dim, t, ws), (-5.0,),
        cpu_rows=cpu_rows, total_rows=lengths[0], scratch_bytes=ws, launches_per_step=3, roofline_note=KDA_ROOFLINE_NOTE)


WORKLOADS = {
    "mamba2_chunk_scan_paper": lambda w, r: _mamba2_workload(),
    "mamba2_chunk_scan_b8_l8192": lambda w, r: _mamba2_workload(8, 8192, 16),
    "attention_causal_4x32x2048x128": lambda w, r: _attention_workload(4, 32, 2048, 128, world=w, rank=r),
    "attention_causal_4x32x512x128": lambda w, r: _attention_workload(4, 32, 512, 128, world=w, rank=r),
    "attention_causal_4x32x8192x128": lambda w, r: _attention_workload(4, 32, 8192, 128, world=w, rank=r),
    "attention_causal_4x32x2048x64": lambda w, r: _attention_workload(4, 32, 2048, 64, world=w, rank=r),
    "bitdelta_base_m1": lambda w, r: _bitdelta_base_workload(1),
    "bitdelta_base_m16": lambda w, r: _bitdelta_base_workload(16),
    "bitdelta_base_m128": lambda w, r: _bitdelta_base_workload(128),
    "kda_gated": lambda w, r: _kda_gated_workload(world=w, rank=r),
    "gemm_nt_4096": lambda w, r: _gemm_nt_workload(4096, 4096, 4096),
    "gemm_nt_8192": lambda w, r: _gemm_nt_workload(8192, 8192, 8192),
    "gemm_nt_512": lambda w, r: _gemm_nt_workload(512, 512, 512),
    "gemm_nt_4095": lambda w, r: _gemm_nt_workload(4095, 4096, 4096),
    "rmsnorm_4096x4096": lambda w, r: _rmsnorm_workload(4096, 4096),
    "rmsnorm_4096x1024": lambda w, r: _rmsnorm_workload(4096, 1024),
    "rmsnorm_4096x8192": lambda w, r: _rmsnorm_workload(4096, 8192),
    "rmsnorm_4093x4096": lambda w, r: _rmsnorm_workload(4093, 4096),
    # The task contracts at their reference paper sizes (tasks/<task>/opspec.json sizes.paper).
    "softmax_8192x2048": lambda w, r: _membound_task_workload("softmax", (8192, 2048), kernel="softmax_vec_kernel"),
    "reduction_sum_4096x4096": lambda w, r: _membound_task_workload("reduction_sum", (4096, 4096), kernel="rowsum_vec_kernel"),
    "rope_2x32x1024x128": lambda w, r: _membound_task_workload("rope", (2, 32, 1024, 128), kernel="rope_vec_kernel"),
    "silu_16777216": lambda w, r: _membound_task_workload("silu", (16777216,), kernel="act_kernel"),
    "swiglu_16777216": lambda w, r: _membound_task_workload("swiglu", (16777216,), kernel="act_kernel"),
    "gemm_nn_2048": lambda w, r: _gemm_nn_task_workload(),
    "bitdelta_gemm_512x4096x4096": lambda w, r: _bitdelta_task_workload(),
    "attention_full_2x8x1024x64": lambda w, r: _attention_workload(2, 8, 1024, 64, causal=False, dtype="fp16", world=w, rank=r),
    "varlen_kda_h64_mixed": lambda w, r: _kda_task_workload(),
    "relu_16777216": lambda w, r: _membound_task_workload("relu", (16777216,), kernel="act_kernel"),
    "sigmoid_16777216": lambda w, r: _membound_task_workload("sigmoid", (16777216,), kernel="act_kernel"),
    "sigmoid_shift_16777216": lambda w, r: _membound_task_workload("sigmoid_shift", (16777216,), kernel="act_kernel"),
    "lion_8388608": lambda w, r: _lion_task_workload(),
    "gemv_4096x4096": lambda w, r: _gemv_task_workload(),
    "gemm_silu_2048": lambda w, r: _gemm_silu_task_workload(),
    "kda_fixed_256x8x64": lambda w, r: _kda_fixed_task_workload(),
}
DEFAULT_WORKLOAD = "gemm_nt_4096"


# ---- helpers --------------------------------------------------------------------------------


def _threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        info = threadpool_info()
        blas = [i for i in info if i.get("user_api") == "blas"]
        if blas:
            return int(blas[0].get("num_threads") or os.cpu_count() or 1)
    except Exception:
        pass
    return os.cpu_count() or 1


def _sample_rows(wl: Workload, seconds: float) -> int:
    """Rows of a CPU sample that takes about ``seconds`` (calibrated on a small sample)."""
    probe = max(1, min(wl.total_rows, 32))
    fn, _, _ = wl.cpu_rows(probe)
    fn()
    t0 = time.perf_counter()
    fn()
    per_row = max((time.perf_counter() - t0) / probe, 1e-9)
    rows = int(seconds / per_row)
    return max(1, min(wl.total_rows, rows))


def cpu_baseline(wl: Workload, budget_s: float = 15.0) -> dict:
    """The oracle port on a bounded row sample of the workload, repeated for about budget_s."""
    threads = _threads()
    rows = _sample_rows(wl, min(2.0, budget_s / 4))
    fn, units, desc = wl.cpu_rows(rows)
    fn()
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 1000:
            break
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    return {"value": units * reps / el / scale, "unit": wl.unit, "cores": threads, "kind": "port",
            "sample": f"{desc} x{reps} in {el:.1f} s"}


# Sample of each configuration's registered-baseline timing (rows / heads / tokens), sized so a
# call takes tens of milliseconds on the host cores.
REGISTERED_SAMPLE = {"rmsnorm": 4096, "gemm_nt": 512, "bitdelta_base": 4096, "attention": 4, "kda_gated": 512}


def registered_baseline(wl: Workload, reps: int = 7) -> dict | None:
    """The task's registered library baseline (``oracle/baselines.py``: the torch calls of
    tasks/<t>/baselines.py on CPU tensors) on a sample of the workload, timed with this
    library's timing protocol (interleaved repetitions, median) on all host threads."""
    import torch

    from oracle import baselines
    from shapeforge_b200 import protocol

    key = next((k for k in REGISTERED_SAMPLE if wl.name.startswith(k)), None)
    if key is None or wl.cpu_inputs is None:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    fn, units, desc = baselines.registered(wl.name, wl.cpu_inputs(), REGISTERED_SAMPLE[key])

    def run_k(k: int) -> float:
        t0 = time.perf_counter()
        for _ in range(k):
            fn()
        return time.perf_counter() - t0

    noise, stats, attempts = protocol.measure_interleaved({"registered": run_k}, reps=reps, kmin=1, target_s=0.05)
    per = stats["registered"].median_s
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    return {"value": units / per / scale, "unit": wl.unit, "cores": threads, "kind": "registered baseline (torch CPU)",
            "sample": f"{desc}: median of {stats['registered'].reps} repetitions, {per * 1e3:.2f} ms per call, CV {noise:.3f}"}


def _traffic(kernel: str, workload: str) -> float | None:
    """Per-launch DRAM traffic recorded from an ncu capture in profiles/ (``traffic_bytes: N``)."""
    for p in sorted((ROOT / "profiles").glob("*.md")):
        text = p.read_text(errors="replace")
        if f"kernel: {kernel}" in text and f"workload: {workload}" in text:
            for line in text.splitlines():
                if line.strip().startswith("traffic_bytes_per_launch:"):
                    try:
                        return float(line.split(":", 1)[1].strip())
                    except ValueError:
                        return None
    return None


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---- arms -----------------------------------------------------------------------------------


def run_reference(args, wl: Workload) -> dict:
    """Each step runs the oracle port once on a row sample sized so W + K steps take about a minute."""
    threads = _threads()
    per_step_s = max(0.005, 60.0 / (args.steps + args.warmup))
    rows = _sample_rows(wl, per_step_s)
    fn, units, desc = wl.cpu_rows(rows)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    el = time.perf_counter() - t0
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    value = units * args.steps / el / scale
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": wl.unit,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": wl.dtype,
        "data": "synthetic",
        "config": _config(wl, args.gpus),
        "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": "port",
                         "sample": f"{desc} per step (oracle/ restatement of the task reference.py)"},
        "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# The naturally sharded paths, measured beside the default (replicated) workload so that a run at
# --gpus N also reports them: attention split by (b, h), varlen KDA by (sequence, head) chains.
SHARDED_WORKLOADS = ("attention_causal_4x32x2048x128", "kda_gated")


def _peak(wl: Workload, clock_summary: dict | None) -> tuple[float, str]:
    peaks, peak_src = measured_peaks()
    if wl.bound == "tensor":
        # The burst GEMM peak for a kernel that ran at full clock; the sustained one (measured
        # under the power cap) when the timed region itself was power-capped or clocked down.
        capped = bool(clock_summary) and ("sw_power_cap" in clock_summary["reasons"] or
                                          clock_summary["sm_mhz"] < 0.97 * float(clock_summary["sm_max_mhz"] or 0))
        kind = "bf16_tflops_sustained" if capped else "bf16_tflops"
    else:
        kind = "hbm_gbs"
    return float(peaks.get(kind, FALLBACK_PEAKS[kind])), f"{peak_src} ({kind})"


def _device_timed(args, wl: Workload, world: int, local: int, steps: int):
    """W warm-up then exactly ``steps`` launches of ``wl`` (one CUDA graph), bracketed by barriers
    and synchronisation; returns (this rank's seconds, the max over ranks, clock summary)."""
    import torch
    import torch.distributed as dist

    from shapeforge_b200 import _native

    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    sets = wl.make_sets(dev, wl.nsets)
    ptr_sets = [p for _, p in sets]
    desc = wl.desc()

    def barrier():
        if world > 1:
            dist.barrier()

    _native.run_batch(desc, ptr_sets, args.warmup, sptr)
    torch.cuda.synchronize(dev)
    # Timed: sf_run_batch captures the launches (set i % nsets for launch i) into one CUDA graph
    # before the timed region, launches it between two CUDA events on this stream and
    # synchronises; it returns the events' elapsed device time.  (--no-graph enqueues the
    # launches one by one from C instead.)
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        el_s = _native.run_batch(desc, ptr_sets, steps, sptr, use_graph=not args.no_graph)
        torch.cuda.synchronize(dev)
    barrier()
    code, where = _native.kernel_status(sptr)
    if code:
        raise RuntimeError(f"tensor-core kernel status {code} (wait {where}) during the timed region")
    t = torch.tensor([el_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return el_s, float(t.item()), clocks.summary(), sets


def run_sharded(args, world: int, rank: int, local: int) -> dict:
    """Device-timed lines of the sharded workloads at this world size (strong scaling: the job is
    the full problem, value = its units / the slowest rank's time)."""
    import torch

    out = {}
    steps = max(1, min(args.steps, 100))
    for name in SHARDED_WORKLOADS:
        wl = WORKLOADS[name](world, rank)
        el_s, max_s, clock_summary, sets = _device_timed(args, wl, world, local, steps)
        del sets
        torch.cuda.empty_cache()
        scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
        job = wl.total_units if wl.sharded else wl.units_per_step
        achieved = wl.units_per_step / (el_s / steps) / scale
        peak, peak_src = _peak(wl, clock_summary)
        out[name] = {
            "value": job * steps / max_s / scale,
            "unit": wl.unit,
            "ms_per_step": max_s / steps * 1e3,
            "steps": steps,
            "scaling": "strong",
            "n_gpus": world,
            "parallelism": wl.shard_note if world > 1 else "1 GPU",
            "roofline": {"bound": wl.bound, "achieved_rank0": achieved, "peak": peak, "frac_rank0": achieved / peak,
                         "peak_source": peak_src, "kernel": wl.kernel},
            "gpu_launches": steps * wl.launches_per_step,
            "clocks": clock_summary,
        }
    return out


def _config(wl: Workload, world: int) -> dict:
    return dict(wl.config, parallelism=(wl.shard_note if wl.sharded else f"replicas x{world}") if world > 1 else "1 GPU")


def run_ours(args, wl: Workload, world: int, rank: int, local: int) -> dict | None:
    import torch
    import torch.distributed as dist

    from shapeforge_b200 import _native

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    _native.load()
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    # W untimed warm-up steps, then exactly K timed steps (one CUDA graph between two events).
    el_s, max_s, clock_summary, sets = _device_timed(args, wl, world, local, args.steps)
    del sets

    # End to end through the C ABI with host buffers (pinned): every step copies its inputs from
    # host to device, runs the operator and copies its outputs back, all inside the timed region.
    # Steps are pipelined over two buffer sets and three streams (host->device, compute,
    # device->host), so the copies of one step overlap the kernel and copies of its neighbours.
    h_in, out_specs = wl.host_inputs()
    d_in = [[h.to(dev) for h in h_in] for _ in range(2)]
    d_out = [[torch.empty(shape, dtype=dt, device=dev) for shape, dt in out_specs] for _ in range(2)]
    h_out = [[torch.empty(shape, dtype=dt).pin_memory() for shape, dt in out_specs] for _ in range(2)]
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    e2e_steps = max(1, min(args.steps, 50))

    def run_e2e(n_steps):
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for st in (s_in, s_cmp, s_out):
            st.wait_event(start)
        in_done, cmp_done, out_done = [], [], []
        for i in range(n_steps):
            b = i % 2
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(cmp_done[i - 2])  # the kernel of step i-2 has read d_in[b]
                for d, h in zip(d_in[b], h_in):
                    d.copy_(h, non_blocking=True)
                in_done.append(torch.cuda.Event())
                in_done[-1].record(s_in)
            s_cmp.wait_event(in_done[i])
            if i >= 2:
                s_cmp.wait_event(out_done[i - 2])  # d_out[b] has been copied out
            wl.e2e_launch(d_in[b], d_out[b], s_cmp.cuda_stream)
            cmp_done.append(torch.cuda.Event())
            cmp_done[-1].record(s_cmp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(cmp_done[i])
                for h, d in zip(h_out[b], d_out[b]):
                    h.copy_(d, non_blocking=True)
                out_done.append(torch.cuda.Event())
                out_done[-1].record(s_out)
        for st in (s_in, s_cmp, s_out):
            ev = torch.cuda.Event()
            ev.record(st)
            stream.wait_event(ev)
        stop.record(stream)
        stop.synchronize()
        return start.elapsed_time(stop) * 1e-3

    run_e2e(2)
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    e2e_s = torch.tensor([run_e2e(e2e_steps)], dtype=torch.float64, device=dev)
    torch.cuda.synchronize(dev)
    barrier()
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_time = float(e2e_s.item())
    h_out = h_out[0]

    if rank != 0:
        return None

    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    job_units = wl.total_units if wl.sharded else world * wl.units_per_step
    value = job_units * args.steps / max_s / scale
    # Algorithmic units of one step over the step's device time (one launch of the dominant kernel).
    per_step_s = el_s / args.steps
    achieved = wl.units_per_step / per_step_s / scale
    peak, peak_src = _peak(wl, clock_summary)
    e2e_value = job_units * e2e_steps / e2e_time / scale
    h2d = sum(h.numel() * h.element_size() for h in h_in)
    d2h = sum(h.numel() * h.element_size() for h in h_out)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": wl.unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": max_s / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if wl.sharded else "weak",
        "vs_baseline": None,
        "dtype": wl.dtype,
        "data": "synthetic",
        "config": _config(wl, world),
        "roofline": {
            "bound": wl.bound,
            "achieved": achieved,
            "peak": peak,
            "unit": wl.unit,
            "frac": achieved / peak,
            "peak_source": peak_src,
            "traffic": _traffic(wl.kernel, wl.name),
            "kernel": wl.kernel,
            **({"note": wl.roofline_note} if wl.roofline_note else {}),
        },
        "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps,
                "path": "sf_* C ABI, pinned host buffers, H2D + kernel + D2H per step, consecutive steps pipelined over two buffer sets"},
        "gpu_launches": args.steps * wl.launches_per_step,
        "clocks": clock_summary,
        "impl": "ours",
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl)
        reg = registered_baseline(wl)
        if reg is not None:
            line["registered_baseline"] = reg
    return line


def _finish(args, line: dict | None, world: int, rank: int, local: int) -> dict | None:
    """Add the sharded paths' lines to the default workload's line (every rank takes part)."""
    if args.workload == DEFAULT_WORKLOAD and not args.no_sharded:
        sharded = run_sharded(args, world, rank, local)
        if line is not None:
            line["sharded"] = sharded
            line["gpu_launches"] += sum(v["gpu_launches"] for v in sharded.values())
    return line


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--variant", type=int, default=0,
                    help="forced kernel variant of an operator workload (sf_op_desc.variant; 0 = default dispatch)")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the sharded attention / KDA lines added to the default workload's line")
    ap.add_argument("--no-graph", action="store_true",
                    help="enqueue the K timed launches one by one instead of as one captured CUDA graph")
    args = ap.parse_args()
    global VARIANT
    VARIANT = args.variant
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, rank, local = _dist()
    wl = WORKLOADS[args.workload](world, rank)

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, wl)), flush=True)
        return

    if world > 1:
        import datetime

        # Communicator set-up lines (ranks, transports, NVLS) go to stderr, whatever the
        # environment asked for; stdout keeps the one JSON line.
        os.environ["NCCL_DEBUG"] = "INFO"
        os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
        os.environ["NCCL_DEBUG_FILE"] = "/dev/stderr"
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        line = _finish(args, run_ours(args, wl, world, rank, local), world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
