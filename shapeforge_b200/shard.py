"""Partitioning the naturally sharded operators over the GPUs of one node.

Flash attention is independent per (batch, head): one process per GPU takes a contiguous range of
the B*H heads and runs the same kernel on its slice.  Varlen KDA is independent per (sequence,
head) chain, and chains differ in length, so they are dealt to ranks by a longest-processing-time
balance over their token counts (``chain_assign``); each rank repacks its chains as single-head
sequences of one packed batch (``pack_chains``: H = 1, one CTA per chain as before), so any subset
of chains runs through the unchanged kernel.  Neither path has a collective on the data path; the
outputs (and KDA's final states) are gathered with NCCL all-gathers (``torch.distributed`` over
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


# ---- varlen KDA: (sequence, head) chains ------------------------------------------------------------


def chain_assign(lengths: Sequence[int], heads: int, world: int) -> list[list[tuple[int, int]]]:
    """Deal the ``len(lengths) * heads`` chains to ``world`` ranks, longest first, each to the rank
    with the fewest tokens so far (``lpt_assign`` over token counts).  Each rank's list is sorted
    by (sequence, head); empty sequences are dealt too (they cost nothing)."""
    chains = [(s, h) for s in range(len(lengths)) for h in range(heads)]
    parts = lpt_assign([float(lengths[s]) for s, _ in chains], world)
    return [[chains[i] for i in part] for part in parts]


def chain_offsets(cu_seqlens: Sequence[int], chains: Sequence[tuple[int, int]]) -> list[int]:
    """cu_seqlens of the packed batch whose sequences are ``chains`` in order."""
    out = [0]
    for s, _ in chains:
        out.append(out[-1] + int(cu_seqlens[s + 1]) - int(cu_seqlens[s]))
    return out


def pack_chains(t: torch.Tensor, cu_seqlens: Sequence[int], chains: Sequence[tuple[int, int]]) -> torch.Tensor:
    """Rows of ``t`` [T, H, ...] for each chain (its sequence's tokens, its head), concatenated
    into [T_r, 1, ...]: the chains become the sequences of a single-head packed batch."""
    parts = [t[int(cu_seqlens[s]):int(cu_seqlens[s + 1]), h:h + 1] for s, h in chains]
    if not parts:
        return t[:0, :1].contiguous()
    return torch.cat(parts, dim=0).contiguous()


def pack_states(state: torch.Tensor, chains: Sequence[tuple[int, int]]) -> torch.Tensor:
    """Per-chain rows of a state tensor [N, H, ...] as [n_r, 1, ...]."""
    if not chains:
        return state[:0, :1].contiguous()
    return torch.stack([state[s, h:h + 1] for s, h in chains]).contiguous()


def unpack_chains(packed: torch.Tensor, cu_seqlens: Sequence[int], chains: Sequence[tuple[int, int]], out: torch.Tensor) -> None:
    """Scatter a packed [T_r, 1, ...] result back into ``out`` [T, H, ...] (inverse of pack_chains)."""
    offs = chain_offsets(cu_seqlens, chains)
    for i, (s, h) in enumerate(chains):
        out[int(cu_seqlens[s]):int(cu_seqlens[s + 1]), h] = packed[offs[i]:offs[i + 1], 0]


def unpack_states(packed: torch.Tensor, chains: Sequence[tuple[int, int]], out: torch.Tensor) -> None:
    """Scatter per-chain states [n_r, 1, ...] back into ``out`` [N, H, ...]."""
    for i, (s, h) in enumerate(chains):
        out[s, h] = packed[i, 0]


def _gather_rows(local: torch.Tensor, counts: Sequence[int], group=None) -> list[torch.Tensor]:
    """All-gather tensors whose first dimension differs by rank (padded to the largest)."""
    import torch.distributed as dist

    width = max(max(counts), 1)
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in counts]
    dist.all_gather(parts, pad, group=group)
    return [p[:n] for p, n in zip(parts, counts)]


def sharded_chains(fn: Callable[..., tuple[torch.Tensor, torch.Tensor]], tensors: Sequence[torch.Tensor], cu_seqlens: Sequence[int],
                   heads: int, state0: torch.Tensor | None = None, group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Run ``fn(*packed tensors, packed cu_seqlens, packed state0 or None)`` on this rank's chains
    and all-gather.

    ``tensors`` are token-major [T, H, ...] (q, k, v, g, beta); ``state0`` is [N, H, Dv, Dk] or None;
    ``fn`` returns (output [T_r, 1, Dv], final states [n_r, 1, Dv, Dk]) for the packed batch.
    Returns the full (output [T, H, Dv], final states [N, H, Dv, Dk]) on every rank."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    parts = chain_assign([int(cu_seqlens[i + 1]) - int(cu_seqlens[i]) for i in range(len(cu_seqlens) - 1)], heads, world)
    mine = parts[rank]
    packed = [pack_chains(t, cu_seqlens, mine) for t in tensors]
    cu_r = torch.tensor(chain_offsets(cu_seqlens, mine), dtype=torch.int32, device=tensors[0].device)
    out_r, fin_r = fn(*packed, cu_r, None if state0 is None else pack_states(state0, mine))
    tokens = [chain_offsets(cu_seqlens, p)[-1] for p in parts]
    outs = _gather_rows(out_r, tokens, group)
    fins = _gather_rows(fin_r, [len(p) for p in parts], group)
    total = int(cu_seqlens[-1])
    out = torch.zeros((total, heads) + tuple(out_r.shape[2:]), dtype=out_r.dtype, device=out_r.device)
    fin = torch.zeros((len(cu_seqlens) - 1, heads) + tuple(fin_r.shape[2:]), dtype=fin_r.dtype, device=fin_r.device)
    for p, o, f in zip(parts, outs, fins):
        unpack_chains(o, cu_seqlens, p, out)
        unpack_states(f, p, fin)
    return out, fin
