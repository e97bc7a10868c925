"""gemm_nt: C = A . B^T with B stored [N, K] -- the dense-gemm workload, a layout variant of
tasks/gemm (whose B is [K, N]).

Oracle: the storage-rounded inputs multiplied in fp64.  Case families: normal N(0,1),
wide_range (sign * 10^U(-3,2)), large U(-4,4), tiny (the format's subnormal/near-normal range),
outlier (N(0,1) with 1e-3 of the entries x100), ieee (normal with NaN/+-Inf/-0 placed in A), and
uniform U(-1,1) (the workload's timing distribution).  Each tensor has its own seed offset.
"""

import math

import torch

_TINY = {"fp16": (2.0 ** -24, 2.0 ** -12), "bf16": (2.0 ** -125, 2.0 ** -113)}
_SPECIALS = (float("nan"), float("inf"), float("-inf"), -0.0)
_OFFSET = {"A": 0, "B": 101}


def _generator(seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    return g


def _draw(case, shape, seed, dtype):
    g = _generator(seed)
    f64 = torch.float64
    if case in ("normal", "ieee"):
        return torch.randn(shape, generator=g, dtype=f64)
    if case == "uniform":
        return torch.rand(shape, generator=g, dtype=f64) * 2.0 - 1.0
    if case == "large":
        return (torch.rand(shape, generator=g, dtype=f64) * 2.0 - 1.0) * 4.0
    if case == "wide_range":
        e = torch.rand(shape, generator=g, dtype=f64) * 5.0 - 3.0
        sign = torch.where(torch.rand(shape, generator=g, dtype=f64) < 0.5, -1.0, 1.0)
        return sign * torch.pow(10.0, e)
    if case == "tiny":
        lo, hi = _TINY[dtype]
        e = torch.rand(shape, generator=g, dtype=f64) * (math.log2(hi) - math.log2(lo)) + math.log2(lo)
        sign = torch.where(torch.rand(shape, generator=g, dtype=f64) < 0.5, -1.0, 1.0)
        return sign * torch.pow(2.0, e)
    if case == "outlier":
        x = torch.randn(shape, generator=g, dtype=f64)
        return torch.where(torch.rand(shape, generator=g, dtype=f64) < 1e-3, x * 100.0, x)
    raise ValueError(f"unknown case {case!r}")


def _place_specials(t, seed):
    flat = t.reshape(-1).clone()
    count = max(2, min(64, flat.numel() // 64))
    pos = torch.randperm(flat.numel(), generator=_generator(seed))[:count]
    pos[0], pos[-1] = 0, flat.numel() - 1
    for i, p in enumerate(pos.tolist()):
        flat[p] = _SPECIALS[i % len(_SPECIALS)]
    return flat.reshape(t.shape)


def gen_inputs(case, seed, instance):
    s = instance.symbols
    m, n, k = int(s["M"]), int(s["N"]), int(s["K"])
    a = _draw(case, (m, k), seed + _OFFSET["A"], instance.dtype)
    b = _draw(case, (n, k), seed + _OFFSET["B"], instance.dtype)
    if case == "ieee":
        a = _place_specials(a, seed + 7)
    return {"A": a, "B": b}


def reference(inputs, attrs):
    return {"C": inputs["A"].double() @ inputs["B"].double().transpose(0, 1)}
