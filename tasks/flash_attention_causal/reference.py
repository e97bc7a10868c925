"""flash_attention_causal: causal softmax(q k^T / sqrt(D)) v over [B, H, S, D] -- the attention
workload, a variant of tasks/flash_attention (non-causal, SM_SCALE attr, D = 64).

Oracle in fp64: scores, a mask keeping key j <= query i, a max-subtracted softmax, the product
with v.  A row whose scores are all NaN yields NaN.  Cases: normal N(0,1), wide_range
(0.1 * sign * 10^U(-3,2)), large U(-6,6), tiny (the format's subnormal/near-normal range),
outlier (N(0,1) with 1e-3 of the entries x5) and ieee (normal with NaN/+-Inf/-0 placed in q).
"""

import math

import torch

_TINY = {"fp16": (2.0 ** -24, 2.0 ** -12), "bf16": (2.0 ** -125, 2.0 ** -113)}
_SPECIALS = (float("nan"), float("inf"), float("-inf"), -0.0)


def _generator(seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    return g


def _draw(case, shape, seed, dtype):
    g = _generator(seed)
    f64 = torch.float64
    if case in ("normal", "ieee"):
        return torch.randn(shape, generator=g, dtype=f64)
    if case == "large":
        return (torch.rand(shape, generator=g, dtype=f64) * 2.0 - 1.0) * 6.0
    if case == "wide_range":
        e = torch.rand(shape, generator=g, dtype=f64) * 5.0 - 3.0
        sign = torch.where(torch.rand(shape, generator=g, dtype=f64) < 0.5, -1.0, 1.0)
        return 0.1 * sign * torch.pow(10.0, e)
    if case == "tiny":
        lo, hi = _TINY[dtype]
        e = torch.rand(shape, generator=g, dtype=f64) * (math.log2(hi) - math.log2(lo)) + math.log2(lo)
        sign = torch.where(torch.rand(shape, generator=g, dtype=f64) < 0.5, -1.0, 1.0)
        return sign * torch.pow(2.0, e)
    if case == "outlier":
        x = torch.randn(shape, generator=g, dtype=f64)
        return torch.where(torch.rand(shape, generator=g, dtype=f64) < 1e-3, x * 5.0, x)
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
    shape = (int(s["B"]), int(s["H"]), int(s["S"]), int(s["D"]))
    out = {name: _draw(case, shape, seed + off, instance.dtype) for name, off in (("q", 0), ("k", 31), ("v", 62))}
    if case == "ieee":
        out["q"] = _place_specials(out["q"], seed + 7)
    return out


def reference(inputs, attrs):
    q, k, v = (inputs[n].double() for n in ("q", "k", "v"))
    s_len, d = q.shape[-2], q.shape[-1]
    scores = (q @ k.transpose(-1, -2)) / math.sqrt(d)
    keep = torch.ones((s_len, s_len), dtype=torch.bool).tril()
    scores = torch.where(keep, scores, torch.tensor(float("-inf"), dtype=torch.float64))
    row_max = scores.amax(dim=-1, keepdim=True)
    # A row max that is NaN must stay NaN (amax propagates it); -inf cannot occur (the diagonal is kept).
    p = torch.exp(scores - row_max)
    p = p / p.sum(dim=-1, keepdim=True)
    return {"o": p @ v}
