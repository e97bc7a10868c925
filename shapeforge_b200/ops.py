"""Torch-facing wrappers of the sm_100a task operators.

Each function takes CUDA tensors laid out as the task's OpSpec declares (row-major,
contiguous), allocates the output if none is given, and enqueues the kernel on the current
torch CUDA stream through the C ABI.  There is no fallback: a CPU tensor, a wrong dtype or a
missing native library raises.
"""

from __future__ import annotations

import torch

from . import _native

_TORCH_DTYPES = {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32", torch.int32: "i32"}


def dtype_name(t: torch.Tensor) -> str:
    try:
        return _TORCH_DTYPES[t.dtype]
    except KeyError as exc:
        raise TypeError(f"unsupported dtype {t.dtype}") from exc


def _check(t: torch.Tensor, name: str, dtype: torch.dtype | None = None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous (row-major)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} has dtype {t.dtype}, expected {dtype}")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """``y = x * rsqrt(mean(x^2, -1) + eps) * w`` (tasks/rmsnorm/reference.py:110-115)."""
    _check(x, "x")
    _check(w, "w", x.dtype)
    hidden = x.shape[-1] if x.dim() else 1
    if w.numel() != hidden:
        raise ValueError(f"w has {w.numel()} elements, expected hidden={hidden}")
    rows = x.numel() // max(hidden, 1)
    if out is None:
        out = torch.empty_like(x)
    _check(out, "out", x.dtype)
    _native.call(
        "sf_rmsnorm",
        x.data_ptr(),
        w.data_ptr(),
        out.data_ptr(),
        rows,
        hidden,
        float(eps),
        _native.DTYPE_CODES[dtype_name(x)],
        _stream(x),
    )
    return out
