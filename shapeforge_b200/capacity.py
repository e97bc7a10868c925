"""L2 capacity (continuous-batching) calls of the varlen tasks: resolved shapes, the ``cu_seqlens``
boundary contract, logical regions and the padding-poison check, and a batching sweep.

Restates the runtime-shape contract of tcenv/taskcontract/runtime_shape.py (module docstring,
``ResolvedShape``, ``workload_profile_for_case``, ``cu_seqlens_problems``, ``padding_problems``):

* a capacity size declares ``capacity = {total_tokens, num_seqs, cu_seqlens_sentinel (< 0),
  padding_poison_byte (1..255)}`` and ``workload_profiles`` (``{id, seq_lens}``); every buffer is
  capacity-sized, so one build serves every batch;
* case ``i`` of the task's case list runs profile ``i % len(profiles)`` with profiles ordered by
  id — a sweep over the cases is a continuous-batching sequence of different totals and counts;
* a call's ``cu_seqlens`` has ``num_seqs + 1`` legal prefix offsets (int32, starting at 0,
  non-decreasing, ending at the resolved total) and every entry after them is the sentinel;
* the logical region is ``output[:total_tokens]`` and ``final_state[:num_seqs]``; every byte of an
  output outside it must still hold the poison byte after the call (the harness poisons the whole
  output before it).

``CapacityBatch`` owns one set of capacity buffers and runs calls of any resolved shape into them
through ``ops.varlen_kda`` (the kernels stop at the first sentinel offset and leave the padding
alone).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Mapping, Sequence

INT32_MAX = 2**31 - 1


class CapacityError(ValueError):
    """A resolved shape or a boundary tensor that breaks the capacity contract."""


@dataclass(frozen=True)
class CapacitySpec:
    total_tokens: int
    num_seqs: int
    sentinel: int
    poison_byte: int
    profiles: tuple[tuple[str, tuple[int, ...]], ...]  # (id, seq_lens), ordered by id

    @classmethod
    def from_size(cls, size_entry: Mapping[str, Any]) -> "CapacitySpec":
        cap = size_entry.get("capacity")
        if not isinstance(cap, Mapping):
            raise CapacityError("the size declares no capacity (it is not an L2 tier)")
        profiles = tuple(sorted((str(p["id"]), tuple(int(x) for x in p["seq_lens"])) for p in size_entry.get("workload_profiles", ())))
        spec = cls(int(cap["total_tokens"]), int(cap["num_seqs"]), int(cap["cu_seqlens_sentinel"]),
                   int(cap["padding_poison_byte"]), profiles)
        if spec.sentinel >= 0:
            raise CapacityError("the cu_seqlens sentinel must be negative")
        if not 1 <= spec.poison_byte <= 255:
            raise CapacityError("the padding poison byte must be in 1..255")
        if not profiles:
            raise CapacityError("a capacity tier needs at least one workload profile")
        for pid, lens in profiles:
            ResolvedShape.of(lens, spec)  # every declared profile must fit the capacity
        return spec

    def profile_for_case(self, cases: Sequence[str], case: str) -> tuple[str, tuple[int, ...]]:
        if case not in cases:
            raise CapacityError(f"case {case!r} is not declared")
        return self.profiles[list(cases).index(case) % len(self.profiles)]


@dataclass(frozen=True)
class ResolvedShape:
    total_tokens: int
    num_seqs: int

    @classmethod
    def of(cls, seq_lens: Sequence[int], spec: CapacitySpec) -> "ResolvedShape":
        lens = [int(x) for x in seq_lens]
        if any(x < 0 for x in lens):
            raise CapacityError(f"negative sequence length in {lens}")
        shape = cls(sum(lens), len(lens))
        if shape.total_tokens < 1:
            raise CapacityError("a varlen call needs at least one token")
        if shape.num_seqs < 1:
            raise CapacityError("a varlen call needs at least one sequence")
        if shape.total_tokens > spec.total_tokens:
            raise CapacityError(f"resolved total_tokens {shape.total_tokens} exceeds the capacity {spec.total_tokens}")
        if shape.num_seqs > spec.num_seqs:
            raise CapacityError(f"resolved num_seqs {shape.num_seqs} exceeds the capacity {spec.num_seqs}")
        return shape

    def logical(self, name: str) -> slice:
        """The compared rows of an output: tokens for ``output``, sequences for ``final_state``."""
        if name == "output":
            return slice(0, self.total_tokens)
        if name == "final_state":
            return slice(0, self.num_seqs)
        raise CapacityError(f"no logical region is declared for {name!r}")


def cu_seqlens(seq_lens: Sequence[int], spec: CapacitySpec) -> list[int]:
    """The capacity-sized boundary of one batch: prefix offsets, then the sentinel."""
    ResolvedShape.of(seq_lens, spec)
    cu = [0]
    for n in seq_lens:
        cu.append(cu[-1] + int(n))
    return cu + [spec.sentinel] * (spec.num_seqs + 1 - len(cu))


def cu_seqlens_problems(cu: Sequence[int], resolved: ResolvedShape, spec: CapacitySpec) -> tuple[str, ...]:
    """Problems of a call's ``cu_seqlens`` (empty when legal)."""
    values = [int(v) for v in cu]
    problems = []
    if len(values) != spec.num_seqs + 1:
        return (f"cu_seqlens carries {len(values)} offsets, the capacity ABI declares {spec.num_seqs + 1}",)
    prefix, tail = values[: resolved.num_seqs + 1], values[resolved.num_seqs + 1:]
    if prefix[0] != 0:
        problems.append(f"cu_seqlens must start at 0, got {prefix[0]}")
    if prefix[-1] != resolved.total_tokens:
        problems.append(f"cu_seqlens prefix must end at the resolved total_tokens ({resolved.total_tokens}), got {prefix[-1]}")
    for i, (a, b) in enumerate(zip(prefix, prefix[1:])):
        if b < a:
            problems.append(f"cu_seqlens must be non-decreasing; sequence {i} ends before it begins ({a} > {b})")
            break
    for i, v in enumerate(tail):
        if v != spec.sentinel:
            problems.append(f"cu_seqlens tail entry {resolved.num_seqs + 1 + i} is {v}, not the sentinel {spec.sentinel}")
            break
    if any(v < 0 or v > INT32_MAX for v in prefix):
        problems.append("every cu_seqlens prefix offset must lie in the int32 domain")
    return tuple(problems)


def resolved_from_cu(cu: Sequence[int], spec: CapacitySpec) -> ResolvedShape:
    """The resolved shape a boundary claims: offsets up to the first sentinel."""
    values = [int(v) for v in cu]
    n = next((i for i, v in enumerate(values) if v == spec.sentinel), len(values))
    if n < 2:
        raise CapacityError("cu_seqlens has fewer than two prefix offsets")
    lens = [b - a for a, b in zip(values[: n - 1], values[1:n])]
    return ResolvedShape.of(lens, spec) if all(x >= 0 for x in lens) else ResolvedShape(values[n - 1], n - 1)


def padding_problems(name: str, tensor: Any, resolved: ResolvedShape, poison_byte: int) -> tuple[str, ...]:
    """Rows of ``tensor`` outside its logical region whose bytes are not all the poison byte."""
    import torch

    rows = tensor.shape[0]
    region = resolved.logical(name)
    pad = tensor[region.stop:rows]
    if pad.numel() == 0:
        return ()
    raw = pad.contiguous().view(torch.uint8).reshape(pad.shape[0], -1)
    bad = (raw != poison_byte).any(dim=1).nonzero().flatten().tolist()
    return tuple(f"{name} padding row {region.stop + r} was written" for r in bad[:4])


class CapacityBatch:
    """One set of capacity-sized buffers for ``varlen_kda``; calls of any resolved shape run into it."""

    def __init__(self, spec: CapacitySpec, heads: int, dim: int, dtype: Any, device: Any) -> None:
        import torch

        self.spec, self.heads, self.dim = spec, heads, dim
        t, s = spec.total_tokens, spec.num_seqs
        self.output = torch.empty((t, heads, dim), dtype=dtype, device=device)
        self.final_state = torch.empty((s, heads, dim, dim), dtype=torch.float32, device=device)
        self.cu = torch.empty((s + 1,), dtype=torch.int32, device=device)

    def poison(self) -> None:
        import torch

        for t in (self.output, self.final_state):
            t.view(-1).view(torch.uint8).fill_(self.spec.poison_byte)

    def run(self, inputs: Mapping[str, Any], seq_lens: Sequence[int] | None = None, *, cu: Sequence[int] | None = None,
            lower_bound: float = -5.0, variant: int = 0, poison: bool = True) -> ResolvedShape:
        """One call: ``inputs`` are capacity-sized (q, k, v, g, beta, A_log, dt_bias, initial_state,
        scale); the boundary is built from ``seq_lens``, or taken as given (``cu``, checked against
        the contract first); outputs land in this batch's buffers."""
        import torch

        from . import ops

        if cu is None:
            resolved = ResolvedShape.of(seq_lens, self.spec)
            cu = cu_seqlens(seq_lens, self.spec)
        else:
            resolved = resolved_from_cu(cu, self.spec)
            problems = cu_seqlens_problems(cu, resolved, self.spec)
            if problems:
                raise CapacityError("; ".join(problems))
        self.cu.copy_(torch.tensor([int(v) for v in cu], dtype=torch.int32))
        if poison:
            self.poison()
        ops.varlen_kda(inputs["q"], inputs["k"], inputs["v"], inputs["g"], inputs["beta"], inputs["A_log"], inputs["dt_bias"],
                       inputs["initial_state"], self.cu, inputs["scale"], lower_bound=lower_bound, output=self.output,
                       final_state=self.final_state, variant=variant)
        return resolved

    def check_padding(self, resolved: ResolvedShape) -> tuple[str, ...]:
        return (padding_problems("output", self.output, resolved, self.spec.poison_byte)
                + padding_problems("final_state", self.final_state, resolved, self.spec.poison_byte))


# ---- the continuous-batching benchmark mixture ---------------------------------------------------

RING_MAX = 64  # rotation sets a timing run may hold (a memory bound, not a measurement choice)


def benchmark_mixture(cases: Sequence[str], rotation: int, *, capacity: bool, ring_max: int = RING_MAX) -> tuple[str, ...]:
    """The case of each timed rotation set (tcenv/backends/metal/v2_runtime.py ``benchmark_mixture``):
    for a capacity tier at least one set per declared case, cycling in declared order (capped at
    ``ring_max``); otherwise every set is the first case."""
    declared = tuple(str(c) for c in cases)
    if not declared:
        raise CapacityError("a benchmark needs at least one declared case")
    count = max(1, int(rotation))
    if not capacity:
        return tuple(declared[0] for _ in range(count))
    count = min(max(count, len(declared)), int(ring_max))
    return tuple(declared[i % len(declared)] for i in range(count))


def mixture_problems(spec: CapacitySpec, cases: Sequence[str], batches: Sequence[Mapping[str, Any]]) -> tuple[str, ...]:
    """Whether timing evidence is the declared continuous-batching sequence (v2_runtime.py
    ``benchmark_mixture_problems``): declared case order from the first case; each batch's resolved
    shape is its case's profile total/count; every batch is the candidate's; every batch carries an
    evaluation-input digest; every declared profile is covered; a declared full-capacity profile is
    timed."""
    declared = tuple(str(c) for c in cases)
    if not batches:
        return ("a capacity benchmark published no continuous-batching mixture",)
    problems: list[str] = []
    seen: set[str] = set()
    full_timed = False
    for i, b in enumerate(batches):
        want = declared[i % len(declared)]
        if str(b.get("case")) != want:
            problems.append(f"batch[{i}] ran case {b.get('case')!r}; the declared order puts {want!r} there")
            continue
        if b.get("provider") != "candidate":
            problems.append(f"batch[{i}] is attributed to {b.get('provider')!r}, not the candidate")
        digest = b.get("evaluation_input_digest")
        if not isinstance(digest, str) or len(digest) != 64:
            problems.append(f"batch[{i}] carries no evaluation_input_digest")
        pid, lens = spec.profile_for_case(declared, want)
        shape = b.get("resolved_shape") or {}
        if (shape.get("total_tokens"), shape.get("num_seqs")) != (sum(lens), len(lens)):
            problems.append(f"batch[{i}] ran [{shape.get('total_tokens')} / {shape.get('num_seqs')}], case {want!r} declares "
                            f"[{sum(lens)} / {len(lens)}]")
        if shape.get("workload_profile_id") != pid:
            problems.append(f"batch[{i}] names profile {shape.get('workload_profile_id')!r}, not {pid!r}")
        seen.add(pid)
        full_timed |= (sum(lens), len(lens)) == (spec.total_tokens, spec.num_seqs)
    missing = sorted({pid for pid, _ in spec.profiles} - seen)
    if missing:
        problems.append(f"the mixture does not time the declared profiles {missing}")
    declares_full = any((sum(l), len(l)) == (spec.total_tokens, spec.num_seqs) for _, l in spec.profiles)
    if declares_full and not full_timed:
        problems.append("the declared full-capacity profile was not timed")
    return tuple(problems)


def input_digest(inputs: Mapping[str, Any], cu: Sequence[int]) -> str:
    """sha256 over the input bytes (ABI order of ``inputs``) and the boundary."""
    import hashlib

    import torch

    h = hashlib.sha256()
    for name, t in inputs.items():
        h.update(name.encode())
        h.update(t.detach().contiguous().view(-1).view(torch.uint8).cpu().numpy().tobytes())
    h.update(bytes(str([int(v) for v in cu]), "ascii"))
    return h.hexdigest()


def time_mixture(batch: CapacityBatch, spec: CapacitySpec, cases: Sequence[str], inputs_for: Any, *,
                 rotation: int = 0, reps: int = 20, lower_bound: float = -5.0) -> list[dict[str, Any]]:
    """Time the continuous-batching mixture on one set of capacity buffers: set ``i`` runs case
    ``i % len(cases)`` with ``inputs_for(case) -> (inputs, cu)``; each set is the median of ``reps``
    CUDA-event-timed calls.  Returns the ``batches`` evidence ``mixture_problems`` checks."""
    import statistics

    import torch

    out = []
    for case in benchmark_mixture(cases, rotation or len(cases), capacity=True):
        inputs, cu = inputs_for(case)
        resolved = batch.run(inputs, cu=cu, lower_bound=lower_bound)
        pid, _ = spec.profile_for_case(cases, case)
        times = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            batch.run(inputs, cu=cu, lower_bound=lower_bound, poison=False)
            b.record()
            b.synchronize()
            times.append(a.elapsed_time(b) * 1e3)
        out.append({"case": case, "provider": "candidate", "evaluation_input_digest": input_digest(inputs, cu),
                    "resolved_shape": {"total_tokens": resolved.total_tokens, "num_seqs": resolved.num_seqs,
                                       "workload_profile_id": pid},
                    "device_us": float(statistics.median(times))})
    return out
