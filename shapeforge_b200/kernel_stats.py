"""Compiled-kernel resources, the B200 occupancy they allow, and the ABI / limit checks on them.

The reference's Backend protocol asks a backend for the statistics of each compiled pipeline
(``pipeline_stats`` / ``pipeline_stats_many``, tcenv/backends/base.py:305-325; the Metal backend
reports maximum threads per threadgroup, execution width and static threadgroup memory from the
compiled pipeline, tcenv/backends/metal/profile.py:150-230) and for a check of the compiled
artifacts against the target's limits (``check_abi``, base.py:293).  A CUDA cubin's equivalents
are the resources ptxas assigned to each ``extern "C"`` entry — registers per thread, static
shared memory, stack, spills, named barriers — which ``nvcc -Xptxas -v`` prints while the
candidate is built (:func:`parse_ptxas`; the build records them beside the cached cubin).

From those and a launch stage (threads, grid, dynamic shared memory) this module derives the
sm_100 residency per SM — 64K registers allocated per warp in 256-register units, 2048 threads /
64 warps, 32 CTAs, 228 KiB of shared memory with 1 KiB reserved per CTA — and flags what makes a
launch fail (a CTA that needs more registers or shared memory than an SM has, more than 1024
threads, more dynamic shared memory than the target allows) or run badly (spills, a grid below
one wave, a partial last wave).  The live device's occupancy API gives the final word on the GPU
(``sf::resident_ctas`` in the kernels' launchers); this is the host-side reading the evaluator can
make before anything launches.
"""

from __future__ import annotations

import math
import re
from dataclasses import asdict, dataclass
from typing import Any, Iterable, Mapping, Sequence

REGS_PER_SM = 65536
REG_ALLOC_UNIT = 256  # registers, per warp
MAX_REGS_PER_THREAD = 255
MAX_THREADS_PER_SM = 2048
MAX_WARPS_PER_SM = 64
MAX_CTAS_PER_SM = 32
SMEM_PER_SM = 233472  # 228 KiB
SMEM_RESERVED_PER_CTA = 1024
MAX_SMEM_PER_CTA = 232448  # 227 KiB opt-in
MAX_THREADS_PER_CTA = 1024
WARP = 32
SM_COUNT = 148

STATIC_SMEM_LIMIT = "static shared memory above the per-CTA limit"


@dataclass(frozen=True)
class KernelResources:
    """What ptxas assigned to one entry function."""

    name: str
    registers: int
    static_smem: int = 0
    stack_bytes: int = 0
    spill_stores: int = 0
    spill_loads: int = 0
    barriers: int = 0

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


_ENTRY = re.compile(r"Compiling entry function '([^']+)' for 'sm_\w+'")
_FRAME = re.compile(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads")
_USED = re.compile(r"Used (\d+) registers(?:, used (\d+) barriers)?(?:, (\d+) bytes smem)?")


def parse_ptxas(text: str) -> dict[str, KernelResources]:
    """Entry name -> resources from ``-Xptxas -v`` output (one ``Compiling entry function`` block
    per kernel; device functions and the module's global-memory line are ignored)."""
    out: dict[str, KernelResources] = {}
    name: str | None = None
    frame = (0, 0, 0)
    for line in text.splitlines():
        m = _ENTRY.search(line)
        if m:
            name, frame = m.group(1), (0, 0, 0)
            continue
        if name is None:
            continue
        m = _FRAME.search(line)
        if m:
            frame = (int(m.group(1)), int(m.group(2)), int(m.group(3)))
            continue
        m = _USED.search(line)
        if m:
            out[name] = KernelResources(name, int(m.group(1)), int(m.group(3) or 0), frame[0], frame[1], frame[2],
                                        int(m.group(2) or 0))
            name = None
    return out


def resident_ctas(res: KernelResources, threads: int, dynamic_smem: int = 0) -> dict[str, int]:
    """CTAs of ``threads`` threads one sm_100 SM holds at once, and which resource bounds it
    (``limit``: threads / registers / shared_memory / ctas; 0 CTAs when one does not fit)."""
    warps = -(-int(threads) // WARP)
    regs_per_warp = -(-max(int(res.registers), 1) * WARP // REG_ALLOC_UNIT) * REG_ALLOC_UNIT
    by = {
        "threads": MAX_WARPS_PER_SM // warps if warps else 0,
        "registers": (REGS_PER_SM // regs_per_warp) // warps if warps else 0,
        "ctas": MAX_CTAS_PER_SM,
    }
    smem = int(res.static_smem) + int(dynamic_smem)
    by["shared_memory"] = SMEM_PER_SM // (smem + SMEM_RESERVED_PER_CTA) if smem else MAX_CTAS_PER_SM
    limit = min(by, key=lambda k: (by[k], k != "registers"))
    return {"ctas": max(0, min(by.values())), "limit": limit, **{f"by_{k}": v for k, v in by.items()}}


def _count(dims: Any) -> int:
    if isinstance(dims, int):
        return dims
    return int(math.prod(int(d) for d in dims))


def stage_problems(res: KernelResources | None, stage: Any, *, max_threads: int = MAX_THREADS_PER_CTA,
                   max_smem: int = MAX_SMEM_PER_CTA) -> list[str]:
    """Why ``stage`` (``.kernel``, ``.threads``, ``.smem``) cannot launch with ``res``."""
    kernel = getattr(stage, "kernel", "?")
    if res is None:
        return [f"stage `{kernel}` was not compiled (no such extern \"C\" __global__ entry)"]
    threads = _count(stage.threads)
    dyn = int(getattr(stage, "smem", 0) or 0)
    problems = []
    if threads > max_threads:
        problems.append(f"stage `{kernel}` launches {threads} threads per CTA, above the limit of {max_threads}")
    if res.static_smem > max_smem:
        problems.append(f"stage `{kernel}`: {STATIC_SMEM_LIMIT} ({res.static_smem} > {max_smem} bytes)")
    elif res.static_smem + dyn > max_smem:
        problems.append(f"stage `{kernel}` needs {res.static_smem} static + {dyn} dynamic bytes of shared memory, "
                        f"above the per-CTA limit of {max_smem}")
    if threads and resident_ctas(res, threads, dyn)["by_registers"] == 0:
        problems.append(f"stage `{kernel}`: {res.registers} registers x {threads} threads do not fit one SM's "
                        f"{REGS_PER_SM} registers (the launch would fail for too many resources)")
    return problems


def check_stages(resources: Mapping[str, KernelResources], stages: Sequence[Any], *,
                 max_threads: int = MAX_THREADS_PER_CTA, max_smem: int = MAX_SMEM_PER_CTA) -> list[str]:
    problems: list[str] = []
    for st in stages:
        for p in stage_problems(resources.get(st.kernel), st, max_threads=max_threads, max_smem=max_smem):
            if p not in problems:
                problems.append(p)
    return problems


def only_static_smem_limit(violations: Iterable[str]) -> bool:
    v = list(violations)
    return len(v) == 1 and STATIC_SMEM_LIMIT in v[0]


def stats(res: KernelResources, stage: Any, device_info: Mapping[str, Any] | None = None) -> dict[str, Any]:
    """One stage's statistics: the protocol's shared keys plus the CUDA resources and residency."""
    info = dict(device_info or {})
    sms = int(info.get("sm_count") or info.get("multiprocessor_count") or SM_COUNT)
    max_smem = int(info.get("max_smem_per_block_optin") or info.get("max_threadgroup_memory_bytes") or MAX_SMEM_PER_CTA)
    threads = _count(stage.threads)
    grid = _count(stage.grid)
    dyn = int(getattr(stage, "smem", 0) or 0)
    occ = resident_ctas(res, threads, dyn)
    regs_per_warp = -(-max(res.registers, 1) * WARP // REG_ALLOC_UNIT) * REG_ALLOC_UNIT
    max_threads = min(MAX_THREADS_PER_CTA, (REGS_PER_SM // regs_per_warp) * WARP)
    wave = occ["ctas"] * sms
    hints = []
    if res.spill_stores or res.spill_loads:
        hints.append(f"{res.spill_stores} bytes of spill stores and {res.spill_loads} of spill loads per thread")
    if occ["ctas"] and grid < sms:
        hints.append(f"grid of {grid} CTAs leaves {sms - grid} of {sms} SMs idle")
    elif wave and grid > wave and grid % wave and grid % wave < wave // 2:
        hints.append(f"last wave holds {grid % wave} of {wave} resident CTAs")
    if occ["ctas"] and occ["ctas"] * threads < 256 and grid >= sms:
        hints.append(f"{occ['ctas'] * threads} resident threads per SM (limited by {occ['limit']})")
    return {
        "max_total_threads_per_threadgroup": max_threads,
        "thread_execution_width": WARP,
        "static_threadgroup_bytes": res.static_smem,
        "max_threadgroup_memory_bytes": max_smem,
        "launch_threads_per_threadgroup": threads,
        "launch_threadgroups": grid,
        "kernel": res.name,
        "registers_per_thread": res.registers,
        "dynamic_shared_bytes": dyn,
        "stack_bytes": res.stack_bytes,
        "spill_bytes": res.spill_stores + res.spill_loads,
        "resident_ctas_per_sm": occ["ctas"],
        "residency_limit": occ["limit"],
        "waves": (grid / wave) if wave else None,
        "hints": hints,
    }


def stats_many(pairs: Sequence[tuple[KernelResources, Any]], device_info: Mapping[str, Any] | None = None) -> dict[str, Any]:
    """Stage statistics of a multi-stage launch: the single-stage keys over all stages (fewest
    threads, most static memory, the last stage's launch) and ``stages``, one entry per stage."""
    parts = [stats(res, st, device_info) for res, st in pairs]
    if not parts:
        raise ValueError("no stages")
    out = dict(parts[-1])
    out["max_total_threads_per_threadgroup"] = min(p["max_total_threads_per_threadgroup"] for p in parts)
    out["static_threadgroup_bytes"] = max(p["static_threadgroup_bytes"] for p in parts)
    out["registers_per_thread"] = max(p["registers_per_thread"] for p in parts)
    out["spill_bytes"] = sum(p["spill_bytes"] for p in parts)
    out["hints"] = [f"{p['kernel']}: {h}" for p in parts for h in p["hints"]]
    out["stages"] = parts
    return out
