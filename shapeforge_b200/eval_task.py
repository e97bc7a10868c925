"""Evaluate one CUDA candidate on one OpSpec v2 task: the B200 form of ``tcenv.cli eval-v2``.

The reference's command (tcenv/cli.py:69-99 -> cli_common.py:126 ``cmd_eval_v2``) binds the
task, builds the candidate, and — in a supervised worker — runs the declared correctness cases and
optionally the timing (tcenv/backends/metal/v2_runtime.py:331-424 ``prepare_v2_case`` for each
case, then the guarded three-trial check and the interleaved benchmark).  Its v2 runtime is Metal
code, so this module is that path for the CUDA backend, from the same task directory:

* the task's ``opspec.json`` gives the ABI tensors (dims over the size's symbols, ``T`` = the
  instance dtype), the attributes' defaults, the case names, the tolerances and ``exact``;
* the task's own ``reference.py`` gives each case's inputs, ``gen_inputs(case, seed, instance)``
  with seed ``seed + 7919·(i+1)`` for case *i* (v2_runtime.py:1602), rounded to their storage
  dtype, and the fp64 reference ``reference(inputs, attrs)`` on the rounded inputs; the error
  scale is the task's ``error_scale`` hook where it has one, else the RMS of the finite reference;
* the candidate goes through :class:`~shapeforge_b200.track_factory.CudaTrackEvaluator` (nvcc
  build, compiled-resource check, guarded trials, interleaved timing with ``--timed``), by default
  inside a supervised worker (:func:`shapeforge_b200.supervise.run_bounded`) so that a stuck
  compile or launch ends as ``timeout``.

The kernel's arguments are the ABI tensors in order, then the symbols in ``spec_params`` order as
``long long`` (the convention of the portfolio variants).  The report is printed as one JSON
document: ``status`` (``ok`` / ``incorrect`` / ``unsafe`` / ``compile_error`` / ``abi_error`` /
``runtime_error`` / ``timeout`` / ``crash``), per-case summaries, the build, the stage statistics
and, when timed, the timing.
"""

from __future__ import annotations

import argparse
import ctypes
import importlib.util
import json
from pathlib import Path
from types import SimpleNamespace
from typing import Any, Mapping, Sequence

from . import expr
from . import portfolio_pack as pp

CASE_SEED_STRIDE = 7919
SEARCH_SEED = 7


def load_reference(task_dir: str | Path):
    """The task's ``reference.py`` as a module (the task's own input generator and oracle)."""
    path = Path(task_dir) / "reference.py"
    spec = importlib.util.spec_from_file_location(f"sf_task_reference_{abs(hash(str(path.resolve())))}", path)
    if spec is None or spec.loader is None:
        raise FileNotFoundError(path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class Instance:
    """What a task's ``gen_inputs`` / ``error_scale`` read: dtype, symbols, attributes, tolerances,
    each tensor's shape and, for a varlen size with a declared batch, its sequence lengths and
    offsets (``None`` for an L2 capacity size, whose batch the capacity runner resolves)."""

    def __init__(self, opspec: Mapping[str, Any], dtype: str, names: Mapping[str, int],
                 attrs: Mapping[str, float] | None = None, size_entry: Mapping[str, Any] | None = None) -> None:
        self.dtype = dtype
        self.symbols = dict(names)
        lens = (size_entry or {}).get("seq_lens")
        self.canonical_seq_lens = tuple(int(x) for x in lens) if isinstance(lens, list) else None
        self.cu_seqlens = None
        if self.canonical_seq_lens is not None:
            cu = [0]
            for n in self.canonical_seq_lens:
                cu.append(cu[-1] + n)
            self.cu_seqlens = tuple(cu)
        defaults = {k: v.get("default") for k, v in (opspec.get("attrs") or {}).items()}
        self.resolved_attrs = {**defaults, **dict(attrs or {})}
        tol = opspec["numerics"]["tolerances"][dtype]
        self.tolerances = SimpleNamespace(rtol=float(tol["rtol"]), atol_rel=float(tol["atol_rel"]))
        self._tensors = opspec["tensors"]

    def tensor(self, name: str) -> SimpleNamespace:
        t = self._tensors[name]
        return SimpleNamespace(shape=tuple(int(expr.evaluate_term(d, self.symbols)) for d in t["dims"]), dtype=t["dtype"])


def _numpy(t) -> Any:
    import numpy as np

    return np.asarray(t.detach().cpu().double().numpy() if hasattr(t, "detach") else t, dtype=np.float64)


def prepare(task_dir: str | Path, dtype: str, size: str, *, seed: int = SEARCH_SEED, cases: Sequence[str] | None = None,
            attrs: Mapping[str, float] | None = None) -> dict[str, Any]:
    """Specs, cases, tolerances and scalars of one (task, dtype, size): the request without the source."""
    import torch

    from . import compare
    from .runtime import TensorSpec

    opspec = pp.load_opspec(task_dir)
    points = [p for p in pp.domain(opspec, dtype, [size])]
    if not points:
        raise ValueError(f"size {size!r} is not declared for dtype {dtype}")
    names = dict(points[0].names)
    inst = Instance(opspec, dtype, names, attrs, opspec["sizes"][size])
    ref = load_reference(task_dir)
    specs = []
    for name, t in opspec["tensors"].items():
        specs.append(TensorSpec(name, inst.tensor(name).shape, pp.storage_dtype(t["dtype"], dtype), t["role"]))
    storage = {s.name: s.dtype for s in specs}
    chosen = list(cases) if cases else list(opspec["cases"]["names"])
    built = []
    for i, case in enumerate(chosen):
        case_seed = seed + CASE_SEED_STRIDE * (i + 1)
        raw = ref.gen_inputs(case, case_seed, inst)
        inputs = {k: (v if torch.is_tensor(v) else torch.as_tensor(v)).to(storage[k]) for k, v in raw.items()}
        outs = ref.reference(inputs, inst.resolved_attrs)
        refs = {k: _numpy(v) for k, v in outs.items()}
        scales = {k: compare.rms_scale(v) for k, v in refs.items()}
        hook = getattr(ref, "error_scale", None)
        if hook is not None:
            for k, v in (hook(inputs, outs, inst, inst.tolerances) or {}).items():
                scales[k] = _numpy(v)
        built.append((case, inputs, refs, scales))
    numerics = opspec["numerics"]
    return {
        "specs": specs, "cases": built, "rtol": inst.tolerances.rtol, "atol_rel": inst.tolerances.atol_rel,
        "exact": bool(numerics.get("exact", False)), "names": names,
        "scalars": [ctypes.c_longlong(int(names[s])) for s in pp.symbol_order(opspec)],
        "output_dtypes": {s.name: dtype if opspec["tensors"][s.name]["dtype"] == "T" else opspec["tensors"][s.name]["dtype"]
                          for s in specs if s.role != "input"},
    }


def evaluate(task_dir: str | Path, source: str, *, dtype: str = "fp16", size: str = "small", timed: bool = False,
             reps: int = 15, seed: int = SEARCH_SEED, cases: Sequence[str] | None = None, heartbeat: Any = None) -> dict[str, Any]:
    """Build and evaluate ``source`` in this process (the worker side); returns the JSON report."""
    from . import track_factory as tf

    req = prepare(task_dir, dtype, size, seed=seed, cases=cases)
    rep = tf.CudaTrackEvaluator().evaluate(tf.EvaluationRequest(source=source, time_reps=reps if timed else 0, **req))
    rep.update(task=str(Path(task_dir).name), dtype=dtype, size=size, seed=seed, mode="full" if timed else "quick")
    return json.loads(json.dumps(rep, default=str))


def main(argv: Sequence[str] | None = None) -> int:
    ap = argparse.ArgumentParser(prog="python -m shapeforge_b200.eval_task",
                                 description="Evaluate one CUDA candidate on one OpSpec v2 task directory.")
    ap.add_argument("task_dir")
    ap.add_argument("kernel", help="the candidate .cu (extern \"C\" __global__ kernels + a taic-launch block)")
    ap.add_argument("--dtype", default="fp16")
    ap.add_argument("--size", default="small")
    ap.add_argument("--cases", nargs="*", default=None, help="case names (default: every declared case)")
    ap.add_argument("--seed", type=int, default=SEARCH_SEED)
    mode = ap.add_mutually_exclusive_group()
    mode.add_argument("--quick", action="store_true", help="correctness only (the default)")
    mode.add_argument("--timed", action="store_true", help="correctness, then the interleaved timing")
    ap.add_argument("--reps", type=int, default=15)
    ap.add_argument("--timeout", type=float, default=600.0, help="whole-evaluation limit (GPU-lock waits excluded)")
    ap.add_argument("--launch-deadline", type=float, default=10.0)
    ap.add_argument("--in-process", action="store_true", help="no supervised worker")
    a = ap.parse_args(argv)
    source = Path(a.kernel).read_text(encoding="utf-8")
    args = {"task_dir": str(Path(a.task_dir).resolve()), "source": source, "dtype": a.dtype, "size": a.size,
            "timed": bool(a.timed), "reps": a.reps, "seed": a.seed, "cases": a.cases}
    if a.in_process:
        rep = evaluate(**args)
    else:
        from .supervise import run_bounded

        rep = run_bounded("shapeforge_b200.eval_task:evaluate", args, timeout=a.timeout, launch_deadline_s=a.launch_deadline)
    print(json.dumps(rep, indent=1, sort_keys=True))
    return 0 if rep.get("status") == "ok" else 1


if __name__ == "__main__":
    raise SystemExit(main())
