"""CUDA renderer of the sem_int int32 block-program documents.

The sem_int tasks (tasks/sem_int_*/reference.py) define each operator by a program document
(``kind: int32-block-program``): element-wise int32 statements over blocks of ``block``
elements, block reductions (``sum``/``min``/``max``), and a final XOR projection plus
``idx & index_mask``.  The reference renders the same document to Triton and MSL
(tasks/sem_int/program.py:329, :413); this module renders it to one CUDA kernel for sm_100a:
one CTA per block, one thread per element, every statement a line of int32 arithmetic.

Arithmetic: kinds in ``rules.wrap_kinds`` wrap to int32 two's complement (done in unsigned
arithmetic, which is defined to wrap in C++), the other kinds stay in range by construction
(arithmetic ``>>``, ``&`` mask then ``%``, selects, block min/max); ``loop`` wraps the product of
every round.  Block reductions use warp shuffles and shared memory and broadcast to every thread.
"""

from __future__ import annotations

import ctypes
from typing import Any

KERNEL_NAME = "sem_int_program"
REGISTERED_WRAP_KINDS = ("bin", "sbin", "shl", "neg", "hash", "loop", "sum")
KINDS = set(REGISTERED_WRAP_KINDS) | {"shr", "mod", "where", "max", "min"}

_PRELUDE = r"""
#include <stdint.h>
__device__ __forceinline__ int wadd(int a, int b) { return (int)((unsigned)a + (unsigned)b); }
__device__ __forceinline__ int wsub(int a, int b) { return (int)((unsigned)a - (unsigned)b); }
__device__ __forceinline__ int wmul(int a, int b) { return (int)((unsigned)a * (unsigned)b); }
__device__ __forceinline__ int wneg(int a) { return (int)(0u - (unsigned)a); }
__device__ __forceinline__ int wshl(int a, int c) { return (int)((unsigned)a << c); }

// Block reductions over BLOCK threads (BLOCK a multiple of 32); every thread gets the result.
template <int BLOCK>
__device__ __forceinline__ int block_sum(int v, int* red) {
    unsigned s = (unsigned)v;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = (int)s;
    __syncthreads();
    unsigned t = 0;
    for (int w = 0; w < BLOCK / 32; ++w) t += (unsigned)red[w];
    return (int)t;
}
template <int BLOCK>
__device__ __forceinline__ int block_min(int v, int* red) {
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    int t = red[0];
    for (int w = 1; w < BLOCK / 32; ++w) t = min(t, red[w]);
    return t;
}
template <int BLOCK>
__device__ __forceinline__ int block_max(int v, int* red) {
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    int t = red[0];
    for (int w = 1; w < BLOCK / 32; ++w) t = max(t, red[w]);
    return t;
}
"""


def _lit(v: int) -> str:
    """An int32 literal for any value of the document's constant range."""
    return f"(int)0x{int(v) & 0xFFFFFFFF:08x}u"


def render_cuda(document: dict, name: str = KERNEL_NAME) -> str:
    """CUDA source of the program: ``extern "C" __global__ void name(x, y, out, K, n)``."""
    if document.get("kind") != "int32-block-program":
        raise ValueError("not an int32-block-program document")
    rules = document["rules"]
    if tuple(sorted(rules["wrap_kinds"])) != tuple(sorted(REGISTERED_WRAP_KINDS)):
        raise ValueError(f"wrap kinds {rules['wrap_kinds']} are not the registered set {REGISTERED_WRAP_KINDS}")
    block = int(document["block"])
    if block % 32 or not 32 <= block <= 1024:
        raise ValueError(f"block {block} must be a multiple of 32 in [32, 1024]")
    hs, ls = int(rules["hash_shift"]), int(rules["loop_shift"])
    mod_mask, index_mask = int(rules["mod_mask"]), int(rules["index_mask"])
    wrap = set(rules["wrap_kinds"])
    lines = []
    for st in document["statements"]:
        kind, dst = st["kind"], st["dst"]
        if kind not in KINDS:
            raise ValueError(f"unknown statement kind {kind!r}")
        a = st.get("a")
        if kind in ("bin", "sbin"):
            b = st["b"] if st.get("b") else _lit(st["const"])
            op = st["op"]
            if op in "+-*":
                fn = {"+": "wadd", "-": "wsub", "*": "wmul"}[op]
                expr = f"{fn}({a}, {b})" if kind in wrap else f"({a} {op} {b})"
            else:
                expr = f"({a} {op} {b})"
        elif kind == "shl":
            expr = f"wshl({a}, {int(st['const'])})"
        elif kind == "shr":
            expr = f"({a} >> {int(st['const'])})"
        elif kind == "mod":
            expr = f"(({a} & {_lit(mod_mask)}) % {_lit(st['const'])})"
        elif kind == "where":
            expr = f"(({a} {st['op']} {st['b']}) ? {st['c']} : {st['d']})"
        elif kind == "neg":
            expr = f"wneg({a})"
        elif kind == "hash":
            expr = f"wmul({a} ^ ({a} >> {hs}), {_lit(st['const'])})"
        elif kind == "loop":
            lines.append(f"    int {dst} = {a};")
            lines.append(f"    #pragma unroll\n    for (int r = 0; r < {int(st['rounds'])}; ++r) "
                         f"{dst} = wadd(wmul({dst}, {_lit(st['const'])}), {st['b']}) ^ ({dst} >> {ls});")
            continue
        elif kind == "sum":
            expr = f"block_sum<{block}>({a}, red)"
        elif kind == "max":
            expr = f"block_max<{block}>({a}, red)"
        else:  # min
            expr = f"block_min<{block}>({a}, red)"
        lines.append(f"    const int {dst} = {expr};")
    final = document["final"]
    res = final[0]
    for n in final[1:]:
        res = f"({res} ^ {n})"
    body = "\n".join(lines)
    return (
        _PRELUDE
        + f"""
extern "C" __global__ void __launch_bounds__({block}) {name}(const int* __restrict__ x, const int* __restrict__ y,
                                                             int* __restrict__ out, int K, int n) {{
    __shared__ int red[{block // 32}];
    const int i = blockIdx.x * {block} + threadIdx.x;
    const int xv = x[i];
    const int yv = y[i];
    const int idx = i;
{body}
    out[i] = wadd({res}, idx & {index_mask});
}}
"""
    )


class SemIntProgram:
    """A compiled, loaded program: ``run(x, y, out, K)`` on int32 CUDA tensors of n = P*block."""

    def __init__(self, document: dict):
        from .candidates import Module, compile_source

        self.document = document
        self.block = int(document["block"])
        self.source = render_cuda(document)
        self.module = Module(compile_source(self.source, name="sem_int"))

    def run(self, x: Any, y: Any, out: Any, k: int, stream: int | None = None) -> None:
        import torch

        n = x.numel()
        if n % self.block:
            raise ValueError(f"N={n} is not a multiple of the block {self.block}")
        if n == 0:
            return
        for t, nm in ((x, "x"), (y, "y"), (out, "out")):
            if not t.is_cuda or t.dtype != torch.int32 or not t.is_contiguous() or t.numel() != n:
                raise ValueError(f"{nm} must be a contiguous int32 CUDA tensor of {n} elements")
        s = torch.cuda.current_stream().cuda_stream if stream is None else stream
        self.module.launch(KERNEL_NAME, (n // self.block,), (self.block,),
                           [x.data_ptr(), y.data_ptr(), out.data_ptr(), ctypes.c_int(int(k)), ctypes.c_int(n)], stream=s)
