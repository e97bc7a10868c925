"""ctypes binding of ``libsfcuda.so`` (declared in ``include/sfcuda.h``).

This is the only module that touches the native library.  It fails loudly: there is no CPU
or eager fallback for any operator, so a missing or unloadable library raises
:class:`NativeUnavailable` at first use.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(os.environ.get("SFCUDA_LIB", Path(__file__).resolve().parent / "libsfcuda.so"))

SF_OK = 0
SF_EINVAL = 2
SF_EDEVICE = 3

DTYPE_CODES = {"fp16": 0, "bf16": 1, "fp32": 2, "i32": 3}

ERR_CAP = 1024


class NativeUnavailable(RuntimeError):
    """``libsfcuda.so`` is missing or failed to load (build it with ``python -m shapeforge_b200.build``)."""


class SfError(RuntimeError):
    """A non-zero status from the C ABI; ``code`` is 2 (invalid arguments) or 3 (device error)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[sfcuda status {code}] {message}")
        self.code = code
        self.message = message


class SfDeviceInfo(ctypes.Structure):
    _fields_ = [
        ("device", ctypes.c_int32),
        ("cc_major", ctypes.c_int32),
        ("cc_minor", ctypes.c_int32),
        ("sm_count", ctypes.c_int32),
        ("global_mem_bytes", ctypes.c_int64),
        ("l2_bytes", ctypes.c_int64),
        ("max_smem_per_block_optin", ctypes.c_int32),
        ("max_threads_per_block", ctypes.c_int32),
        ("clock_khz", ctypes.c_int32),
        ("mem_clock_khz", ctypes.c_int32),
        ("mem_bus_width_bits", ctypes.c_int32),
        ("name", ctypes.c_char * 128),
    ]


class SfOpDesc(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("variant", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("dims", ctypes.c_int64 * 8),
        ("attrs", ctypes.c_double * 4),
    ]


# Operator ids (SF_OP_* in include/sfcuda.h).
OPS = {
    "rmsnorm": 1,
    "gemm_nt": 2,
    "gemm_nn": 3,
    "silu": 4,
    "swiglu": 5,
    "softmax": 6,
    "reduction_sum": 7,
    "rope": 8,
    "bitdelta_gemm": 9,
    "bitdelta_gemm_base": 10,
    "flash_attention": 11,
    "varlen_kda": 12,
    "varlen_kda_gated": 13,
    "mamba2_chunk_scan": 14,
    "relu": 15,
    "sigmoid": 16,
    "sigmoid_shift": 17,
    "lion": 18,
    "gemv": 19,
    "gemm_silu": 20,
    "kda": 21,
}

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64
_F32 = ctypes.c_float
_ERR = (ctypes.c_char_p, _U64)

# name -> (restype, argtypes) for every symbol declared in include/sfcuda.h.
SIGNATURES: dict[str, tuple[object, tuple]] = {
    "sf_version": (ctypes.c_char_p, ()),
    "sf_device_info_get": (ctypes.c_int, (_I32, ctypes.POINTER(SfDeviceInfo), *_ERR)),
    "sf_fill_bytes": (ctypes.c_int, (_P, _U64, _I32, _P, *_ERR)),
    "sf_count_mismatch": (ctypes.c_int, (_P, _U64, _I32, _P, _P, *_ERR)),
    "sf_rmsnorm": (ctypes.c_int, (_P, _P, _P, _I64, _I64, _F32, _I32, _P, *_ERR)),
    "sf_silu": (ctypes.c_int, (_P, _P, _I64, _I32, _P, *_ERR)),
    "sf_swiglu": (ctypes.c_int, (_P, _P, _P, _I64, _I32, _P, *_ERR)),
    "sf_relu": (ctypes.c_int, (_P, _P, _I64, _I32, _P, *_ERR)),
    "sf_sigmoid": (ctypes.c_int, (_P, _P, _I64, _I32, _P, *_ERR)),
    "sf_sigmoid_shift": (ctypes.c_int, (_P, _P, _I64, _I32, _P, *_ERR)),
    "sf_lion": (ctypes.c_int, (_P, _P, _P, _P, _P, _I64, ctypes.c_double, ctypes.c_double, ctypes.c_double, ctypes.c_double, _I32, _P,
                               *_ERR)),
    "sf_gemv": (ctypes.c_int, (_P, _P, _P, _I64, _I64, _I32, _P, *_ERR)),
    "sf_softmax": (ctypes.c_int, (_P, _P, _I64, _I64, _I32, _P, *_ERR)),
    "sf_reduction_sum": (ctypes.c_int, (_P, _P, _I64, _I64, _I32, _P, *_ERR)),
    "sf_rope": (ctypes.c_int, (_P, _P, _I64, _I64, _I64, _I64, ctypes.c_double, _I32, _P, *_ERR)),
    "sf_bitdelta_gemm": (ctypes.c_int, (_P, _P, _P, _I64, _I64, _I64, _F32, _I32, _P, *_ERR)),
    "sf_bitdelta_gemm_base": (ctypes.c_int, (_P, _P, _P, _P, _P, _I64, _I64, _I64, _I32, _P, *_ERR)),
    "sf_flash_attention": (ctypes.c_int, (_P, _P, _P, _P, _I64, _I64, _I64, _I64, _F32, _I32, _I32, _P, *_ERR)),
    "sf_varlen_kda": (ctypes.c_int, (_P,) * 12 + (_I64, _I64, _I64, _F32, _I32, _P, *_ERR)),
    "sf_kda": (ctypes.c_int, (_P,) * 14 + (_I64, _I64, _I64, _F32, _I32, _P, *_ERR)),
    "sf_varlen_kda_gated": (ctypes.c_int, (_P,) * 9 + (_I64, _I64, _I64, _F32, _I32, _P, *_ERR)),
    "sf_varlen_kda_workspace_bytes": (_U64, (_I64, _I64, _I64, _I64)),
    "sf_varlen_kda_ws": (ctypes.c_int, (_P,) * 12 + (_I64, _I64, _I64, _I64, _F32, _I32, _P, _U64, _P, *_ERR)),
    "sf_varlen_kda_gated_workspace_bytes": (_U64, (_I64, _I64, _I64, _I64)),
    "sf_varlen_kda_gated_ws": (ctypes.c_int, (_P,) * 9 + (_I64, _I64, _I64, _I64, _F32, _I32, _P, _U64, _P, *_ERR)),
    "sf_mamba2_chunk_scan": (ctypes.c_int, (_P,) * 8 + (_I64,) * 6 + (_I32, _P, *_ERR)),
    "sf_gemm_nt": (ctypes.c_int, (_P, _P, _P, _I64, _I64, _I64, _I32, _P, *_ERR)),
    "sf_gemm_nn_workspace_bytes": (_U64, (_I64, _I64, _I64, _I32)),
    "sf_gemm_nn": (ctypes.c_int, (_P, _P, _P, _I64, _I64, _I64, _I32, _P, _U64, _P, *_ERR)),
    "sf_gemm_silu": (ctypes.c_int, (_P, _P, _P, _I64, _I64, _I64, _I32, _P, _U64, _P, *_ERR)),
    "sf_gemm_nn_noalloc": (ctypes.c_int, (_P, _P, _P, _I64, _I64, _I64, _I32, _P, *_ERR)),
    "sf_kernel_status": (ctypes.c_int, (ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32), _P, *_ERR)),
    "sf_module_load": (ctypes.c_int, (_P, _U64, ctypes.POINTER(_P), *_ERR)),
    "sf_module_unload": (ctypes.c_int, (_P, *_ERR)),
    "sf_module_get_function": (ctypes.c_int, (_P, ctypes.c_char_p, ctypes.POINTER(_P), *_ERR)),
    "sf_launch_kernel": (
        ctypes.c_int,
        (_P, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
         _P, ctypes.POINTER(_P), *_ERR),
    ),
    "sf_op_nargs": (ctypes.c_int32, (_I32,)),
    "sf_run_op": (ctypes.c_int, (ctypes.POINTER(SfOpDesc), ctypes.POINTER(_P), _U64, _P, *_ERR)),
    "sf_run_batch": (
        ctypes.c_int,
        (ctypes.POINTER(SfOpDesc), ctypes.POINTER(_P), _U64, _U64, _U64, _I32, _P, ctypes.POINTER(ctypes.c_double), *_ERR),
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load (once) and bind the library; raise :class:`NativeUnavailable` if it cannot be loaded."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.is_file():
            raise NativeUnavailable(
                f"{LIB_PATH} is missing; build it with `python -m shapeforge_b200.build` "
                "(there is no CPU fallback for any operator)"
            )
        try:
            lib = ctypes.CDLL(str(LIB_PATH))
        except OSError as exc:
            raise NativeUnavailable(f"cannot load {LIB_PATH}: {exc}") from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name, None)
            if fn is None:
                raise NativeUnavailable(f"{LIB_PATH} does not export {name}")
            fn.restype = restype
            fn.argtypes = list(argtypes)
        _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Call a status-returning entry point; append the error buffer and raise on failure."""
    lib = load()
    buf = ctypes.create_string_buffer(ERR_CAP)
    rc = getattr(lib, name)(*args, buf, ERR_CAP)
    if rc != SF_OK:
        raise SfError(int(rc), buf.value.decode(errors="replace") or name)


def op_desc(op: str, dtype: str, dims=(), attrs=(), variant: int = 0, flags: int = 0) -> SfOpDesc:
    """Build an ``sf_op_desc`` for operator ``op``."""
    d = SfOpDesc()
    d.op = OPS[op]
    d.dtype = DTYPE_CODES[dtype]
    d.variant = int(variant)
    d.flags = int(flags)
    for i, v in enumerate(dims):
        d.dims[i] = int(v)
    for i, v in enumerate(attrs):
        d.attrs[i] = float(v)
    return d


def pointer_array(ptrs) -> ctypes.Array:
    arr = (ctypes.c_void_p * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = int(p)
    return arr


def run_op(desc: SfOpDesc, ptrs, stream: int) -> None:
    arr = pointer_array(ptrs)
    call("sf_run_op", ctypes.byref(desc), arr, len(ptrs), ctypes.c_void_p(stream))


def run_batch(desc: SfOpDesc, sets, iters: int, stream: int, use_graph: bool = False) -> float:
    """Time ``iters`` launches over the rotating argument ``sets``; return device seconds."""
    nargs = len(sets[0])
    flat = [p for s in sets for p in s]
    arr = pointer_array(flat)
    out = ctypes.c_double(0.0)
    call(
        "sf_run_batch",
        ctypes.byref(desc),
        arr,
        nargs,
        len(sets),
        int(iters),
        1 if use_graph else 0,
        ctypes.c_void_p(stream),
        ctypes.byref(out),
    )
    return float(out.value)


def device_info(device: int = 0) -> dict:
    info = SfDeviceInfo()
    call("sf_device_info_get", int(device), ctypes.byref(info))
    out = {name: getattr(info, name) for name, _ in SfDeviceInfo._fields_}
    out["name"] = info.name.decode(errors="replace")
    return out


def kernel_status(stream: int = 0) -> tuple[int, int]:
    """Read and clear the sticky status word of the tensor-core kernels: (code, where)."""
    code = ctypes.c_uint32(0)
    where = ctypes.c_uint32(0)
    call("sf_kernel_status", ctypes.byref(code), ctypes.byref(where), ctypes.c_void_p(stream))
    return int(code.value), int(where.value)


def version() -> str:
    return load().sf_version().decode()
