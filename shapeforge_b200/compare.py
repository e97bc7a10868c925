"""The harness comparator: scaled element error against the fp64 reference.

Restates ``scaled_error`` and ``_floor`` of tcenv/backends/metal/testing.py:140-177 (that
module imports Metal, so it cannot be imported on a CUDA box):

    err = |out - ref| / (rtol * |ref| + atol_rel * scale + floor)

with special values compared exactly — NaN only where the reference is NaN, an infinity of
the same sign where the reference is infinite — a non-finite scale failing everything, and
``exact`` meaning bit equality (integer tasks).  A case passes when every element's error is
at most 1 (``v2_runtime.py:2314-2460``).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

# Smallest positive subnormal of each storage dtype (tcenv/dtypes.py FLOAT_TINY_SUBNORMAL).
TINY_SUBNORMAL = {"fp16": 2.0**-24, "bf16": 2.0**-133, "fp32": 2.0**-149}


def floor_for(dtype: str) -> float:
    """Absolute slack of the output format: half the smallest subnormal spacing (x 1.02)."""
    return 0.51 * TINY_SUBNORMAL.get(dtype, 0.0)


def scaled_error(out, ref, scale, rtol: float, atol_rel: float, exact: bool, floor: float = 0.0) -> np.ndarray:
    """Element-wise normalised error (<= 1 inside tolerance); see the module docstring."""
    o = np.asarray(out, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    if exact:
        return np.where(o != r, np.inf, 0.0)
    scale = np.asarray(scale, dtype=np.float64)
    if not np.isfinite(scale).all():
        return np.full(o.shape, np.inf)
    with np.errstate(all="ignore"):
        tol = rtol * np.abs(r) + atol_rel * scale + floor
        diff = np.abs(o - r)
        same_inf = np.isinf(o) & np.isinf(r) & (np.sign(o) == np.sign(r))
        same_nan = np.isnan(o) & np.isnan(r)
        diff = np.where(same_inf | same_nan, 0.0, diff)
        diff = np.where(np.isnan(diff), np.inf, diff)
        tol = np.nan_to_num(np.maximum(tol, 1e-300), nan=1.0, posinf=1.0)
        return diff / tol


def rms_scale(ref) -> np.float64:
    """Default error scale: RMS of the finite reference (v2_runtime.py:374-381)."""
    r = np.asarray(ref, dtype=np.float64)
    fin = np.where(np.isfinite(r), r, 0.0)
    return np.float64(np.sqrt(np.mean(fin * fin))) if fin.size else np.float64(0.0)


@dataclass
class Verdict:
    ok: bool
    max_err: float
    n_bad: int
    n_elems: int
    nan_count: int
    worst_index: tuple | None
    worst_out: float | None
    worst_ref: float | None

    def summary(self) -> str:
        return (
            f"ok={self.ok} max_scaled_err={self.max_err:.3g} bad={self.n_bad}/{self.n_elems} "
            f"nan={self.nan_count} worst@{self.worst_index}: out={self.worst_out} ref={self.worst_ref}"
        )


def check(out, ref, scale, rtol: float, atol_rel: float, exact: bool = False, dtype: str = "fp16") -> Verdict:
    """Compare ``out`` against ``ref`` and summarise like the reference's CaseResult."""
    o = np.asarray(out, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    if o.shape != r.shape:
        raise ValueError(f"shape mismatch: out {o.shape} vs ref {r.shape}")
    err = scaled_error(o, r, scale, rtol, atol_rel, exact, floor_for(dtype))
    n = int(err.size)
    if n == 0:
        return Verdict(True, 0.0, 0, 0, 0, None, None, None)
    bad = err > 1.0
    flat = int(np.argmax(np.where(np.isnan(err), np.inf, err)))
    idx = np.unravel_index(flat, err.shape)
    return Verdict(
        ok=not bool(bad.any()),
        max_err=float(np.nanmax(err)) if n else 0.0,
        n_bad=int(bad.sum()),
        n_elems=n,
        nan_count=int(np.isnan(o).sum()),
        worst_index=tuple(int(i) for i in idx),
        worst_out=float(o[idx]),
        worst_ref=float(r[idx]),
    )
