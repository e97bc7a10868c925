"""Evidence-bound correctness runs on the B200: guarded buffers and the three trials.

Semantics follow the reference's v2 protocol (tcenv/track/protocol.py:43-143) and correctness
loop (tcenv/backends/metal/v2_runtime.py:1574-1700), with the device side on CUDA:

* every tensor lives inside a larger uint8 allocation with ``GUARD_BYTES`` = 16 KiB bands of
  ``GUARD_PATTERN`` = 0xCD on both sides; a band byte that changed is a safety violation;
* each case runs three trials ``out1``/``out2``/``out3``: inputs are restored from the case's
  bytes every time; pure outputs (and workspaces) are poisoned with ``POISON_PATTERN`` = 0xFF
  (NaN for floats, -1 for integers) for ``out1``/``out3`` and zeroed for ``out2``;
* after each trial: guard bands must be intact, inputs must be unchanged, and the output bytes
  of ``out2``/``out3`` must equal those of ``out1`` (a result that depends on the initial contents
  of an output or workspace is non-deterministic);
* ``out1`` is compared with the fp64 reference by :func:`shapeforge_b200.compare.check` with the
  task tolerances; a case passes when every element's scaled error is <= 1.

The reference outputs and scales are supplied by the caller (the task's own ``reference.py``
through the harness, or any checker); this module never computes a reference.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Mapping, Sequence

import numpy as np
import torch

from . import _native, compare

GUARD_PATTERN = 0xCD
GUARD_BYTES = 16384
POISON_PATTERN = 0xFF
TRIALS = ("out1", "out2", "out3")

RESTORE = "restore_initial"
POISON = "poison"
ZERO = "zero"


@dataclass(frozen=True)
class TensorSpec:
    """One ABI tensor: ``role`` is ``input``, ``output``, ``read_write`` or ``workspace``."""

    name: str
    shape: tuple
    dtype: torch.dtype
    role: str = "input"

    @property
    def nbytes(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n * torch.tensor([], dtype=self.dtype).element_size()


def fill_plan(specs: Sequence[TensorSpec], trial: str) -> dict[str, str]:
    """The fill action of every tensor before a correctness trial (protocol.py:107-143)."""
    if trial not in TRIALS:
        raise ValueError(f"unknown correctness trial {trial!r}; registered trials are {list(TRIALS)}")
    zero = trial == "out2"
    plan = {}
    for s in specs:
        if s.role in ("input", "read_write"):
            plan[s.name] = RESTORE
        elif s.role in ("output", "workspace"):
            plan[s.name] = ZERO if zero else POISON
        else:
            raise ValueError(f"unknown tensor role {s.role!r}")
    return plan


class GuardedBuffer:
    """A device tensor with 0xCD guard bands on both sides."""

    def __init__(self, spec: TensorSpec, device: torch.device):
        self.spec = spec
        self.nbytes = spec.nbytes
        self.raw = torch.empty(self.nbytes + 2 * GUARD_BYTES, dtype=torch.uint8, device=device)
        body = self.raw[GUARD_BYTES : GUARD_BYTES + self.nbytes]
        self.tensor = body.view(spec.dtype).view(spec.shape) if self.nbytes else torch.empty(spec.shape, dtype=spec.dtype, device=device)
        self._stream = torch.cuda.current_stream(device).cuda_stream

    def ptr(self) -> int:
        return self.raw.data_ptr() + GUARD_BYTES

    def fill_guards(self) -> None:
        _native.call("sf_fill_bytes", self.raw.data_ptr(), GUARD_BYTES, GUARD_PATTERN, self._stream)
        _native.call("sf_fill_bytes", self.raw.data_ptr() + GUARD_BYTES + self.nbytes, GUARD_BYTES, GUARD_PATTERN, self._stream)

    def fill(self, value: int) -> None:
        if self.nbytes:
            _native.call("sf_fill_bytes", self.ptr(), self.nbytes, int(value), self._stream)

    def load(self, host: torch.Tensor) -> None:
        if self.nbytes:
            self.tensor.copy_(host.to(self.spec.dtype).reshape(self.spec.shape))

    def guard_hits(self, counter: torch.Tensor) -> int:
        counter.zero_()
        _native.call("sf_count_mismatch", self.raw.data_ptr(), GUARD_BYTES, GUARD_PATTERN, counter.data_ptr(), self._stream)
        _native.call("sf_count_mismatch", self.raw.data_ptr() + GUARD_BYTES + self.nbytes, GUARD_BYTES, GUARD_PATTERN,
                     counter.data_ptr(), self._stream)
        return int(counter.item())

    def bytes(self) -> bytes:
        return self.raw[GUARD_BYTES : GUARD_BYTES + self.nbytes].cpu().numpy().tobytes()


@dataclass
class CaseResult:
    case: str
    ok: bool
    verdicts: dict = field(default_factory=dict)
    safety: list = field(default_factory=list)
    nondeterminism: list = field(default_factory=list)
    kernel_status: tuple = (0, 0)

    def summary(self) -> str:
        parts = [f"{self.case}: ok={self.ok}"]
        for name, v in self.verdicts.items():
            parts.append(f"{name}[{v.summary()}]")
        parts += self.safety + self.nondeterminism
        return " ".join(parts)


class CorrectnessRunner:
    """Runs one operator (``launch(pointers)`` in ABI order) through the three trials per case."""

    def __init__(self, specs: Sequence[TensorSpec], launch: Callable[[list[int]], None], device: torch.device | str = "cuda:0",
                 output_dtypes: Mapping[str, str] | None = None):
        self.device = torch.device(device)
        self.specs = list(specs)
        self.launch = launch
        self.buffers = {s.name: GuardedBuffer(s, self.device) for s in self.specs}
        self.counter = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.output_dtypes = dict(output_dtypes or {})

    def pointers(self) -> list[int]:
        return [self.buffers[s.name].ptr() for s in self.specs]

    def run_case(self, case: str, inputs: Mapping[str, torch.Tensor], refs: Mapping[str, np.ndarray], scales: Mapping[str, object],
                 rtol: float, atol_rel: float, exact: bool = False) -> CaseResult:
        result = CaseResult(case=case, ok=False)
        first: dict[str, bytes] = {}
        for trial in TRIALS:
            plan = fill_plan(self.specs, trial)
            for s in self.specs:
                buf = self.buffers[s.name]
                buf.fill_guards()
                action = plan[s.name]
                if action == RESTORE:
                    buf.load(inputs[s.name])
                elif action == POISON:
                    buf.fill(POISON_PATTERN)
                else:
                    buf.fill(0)
            in_bytes = {s.name: self.buffers[s.name].bytes() for s in self.specs if plan[s.name] == RESTORE and s.role == "input"}
            self.launch(self.pointers())
            torch.cuda.synchronize(self.device)
            result.kernel_status = _native.kernel_status(torch.cuda.current_stream(self.device).cuda_stream)
            if result.kernel_status[0] != 0:
                result.safety.append(f"[{trial}] device wait timed out (status {result.kernel_status})")
            for s in self.specs:
                hits = self.buffers[s.name].guard_hits(self.counter)
                if hits:
                    result.safety.append(f"[{trial}] {s.name}: {hits} guard-band bytes overwritten")
            for name, before in in_bytes.items():
                if self.buffers[name].bytes() != before:
                    result.safety.append(f"[{trial}] input {name} was modified")
            outs = {s.name: self.buffers[s.name].bytes() for s in self.specs if s.role in ("output", "read_write")}
            if trial == "out1":
                first = outs
                for s in self.specs:
                    if s.name in refs:
                        got = self.buffers[s.name].tensor.detach().to(torch.float64).cpu().numpy()
                        dt = self.output_dtypes.get(s.name, _dtype_name(s.dtype))
                        result.verdicts[s.name] = compare.check(got, refs[s.name], scales[s.name], rtol, atol_rel, exact, dt)
            elif outs != first:
                result.nondeterminism.append(
                    f"[{trial}] output differs from out1: it depends on the initial output/workspace contents")
        result.ok = (all(v.ok for v in result.verdicts.values()) and not result.safety and not result.nondeterminism
                     and bool(result.verdicts))
        return result


def _dtype_name(dt: torch.dtype) -> str:
    return {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32"}.get(dt, "fp32")
