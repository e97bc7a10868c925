"""Storage dtype helpers of the oracle (test infrastructure only).

fp16/bf16 tensors are carried as their uint16 bit patterns; these helpers widen them to
float64 exactly and round float values to the storage grid (round-to-nearest-even), the way
``tcenv/tensors.py:25`` ``round_to`` does.
"""

from __future__ import annotations

import numpy as np


def from_storage(bits: np.ndarray, dtype: str) -> np.ndarray:
    """Storage array (uint16 bits for fp16/bf16, native otherwise) -> float64 values."""
    a = np.asarray(bits)
    if dtype == "fp16":
        return a.view(np.float16).astype(np.float64)
    if dtype == "bf16":
        return (a.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    if dtype == "fp32":
        return a.astype(np.float32).astype(np.float64)
    if dtype in ("i32", "u32"):
        return a
    raise ValueError(f"unknown dtype {dtype}")


def to_storage(values: np.ndarray, dtype: str) -> np.ndarray:
    """float values -> storage array, rounding to nearest even (NaN/Inf preserved)."""
    v = np.asarray(values)
    if dtype == "fp16":
        return v.astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        f = v.astype(np.float32)
        u = f.view(np.uint32).astype(np.uint64)
        nan = np.isnan(f)
        rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        return np.where(nan, np.uint16(0x7FC0), rounded).astype(np.uint16)
    if dtype == "fp32":
        return v.astype(np.float32)
    if dtype == "i32":
        return v.astype(np.int32)
    raise ValueError(f"unknown dtype {dtype}")


def round_to(values: np.ndarray, dtype: str) -> np.ndarray:
    """Round to the storage grid and widen back to float64."""
    return from_storage(to_storage(values, dtype), dtype)
