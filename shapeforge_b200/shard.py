"""Partitioning the naturally sharded operators over the GPUs of one node.

Flash attention and varlen KDA are independent per (batch, head) chain, so one process per GPU
takes a contiguous range of heads and runs the same kernel on its slice: no collective on the
data path.  The output shards are gathered with one NCCL all-gather (``torch.distributed``, over
NVLink/NVSwitch) only for the final correctness comparison, outside any timed region.  The dense
operators (rmsnorm, gemm, bitdelta) are not partitioned: each GPU runs whole replicas.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch


def head_ranges(total: int, world: int) -> list[tuple[int, int]]:
    """Contiguous, balanced [start, end) ranges of ``total`` heads over ``world`` ranks."""
    if world < 1:
        raise ValueError("world must be >= 1")
    base, extra = divmod(total, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((start, start + n))
        start += n
    return out


def lpt_assign(costs: Sequence[float], world: int) -> list[list[int]]:
    """Longest-processing-time assignment of independent chains (costs) to ``world`` ranks."""
    loads = [0.0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda j: -costs[j]):
        r = min(range(world), key=lambda q: loads[q])
        parts[r].append(i)
        loads[r] += costs[i]
    return [sorted(p) for p in parts]


def attention_slice(q: torch.Tensor, rank: int, world: int) -> tuple[int, int]:
    """The (b*h) head range of this rank for q [B, H, S, D]."""
    b, h = q.shape[0], q.shape[1]
    return head_ranges(b * h, world)[rank]


def gather_heads(local: torch.Tensor, total_heads: int, group=None) -> torch.Tensor:
    """All-gather per-rank head slices [n_r, ...] into [total_heads, ...] (ranks own contiguous,
    possibly unequal ranges; slices are padded to the largest for the collective)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    ranges = head_ranges(total_heads, world)
    width = max(e - s for s, e in ranges)
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[: e - s] for p, (s, e) in zip(parts, ranges)], dim=0)


def sharded_heads(fn: Callable[..., torch.Tensor], tensors: Sequence[torch.Tensor], total_heads: int, head_dim: int = 0,
                  group=None) -> torch.Tensor:
    """Run ``fn`` on this rank's head range of every tensor (split along ``head_dim``) and
    all-gather the results along that axis."""
    import torch.distributed as dist

    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    s, e = head_ranges(total_heads, world)[rank]
    local = [t.narrow(head_dim, s, e - s).contiguous() for t in tensors]
    out = fn(*local)
    moved = out.movedim(head_dim, 0).contiguous()
    full = gather_heads(moved, total_heads, group)
    return full.movedim(0, head_dim).contiguous()
