"""Seeded correctness-case input streams of the OpSpec tasks (the harness side of ``gen_inputs``).

The adversarial sampler is the frozen G0 block that every migrated task carries
(tasks/rmsnorm/reference.py:12-84: ``_sample`` with the normal / wide_range / large / tiny /
outlier / cancel / const distributions and ``_inject`` planting NaN, +-Inf and -0.0), restated
here on torch's CPU generator so the same seeds give the same tensors as the task modules on
the same torch build.  Per-task magnitudes and seed offsets follow each task's reference.py.
Case seeds follow the harness rule ``seed + 7919 * (case_index + 1)``
(tcenv/backends/metal/v2_runtime.py:1602); the search seed is 7.
"""

from __future__ import annotations

import math

import torch

FLOAT_MAX = {"fp16": 65504.0, "bf16": 3.3895313892515355e38, "fp32": 3.4028234663852886e38}
TINY_NORMAL = {"fp16": 2.0**-14, "bf16": 2.0**-126, "fp32": 2.0**-126}
TINY_SUBNORMAL = {"fp16": 2.0**-24, "bf16": 2.0**-133, "fp32": 2.0**-149}
SPECIALS = (float("nan"), float("inf"), float("-inf"), -0.0)
IEEE_SEED_STRIDE = 104_729
CASE_SEED_STRIDE = 7919
SEARCH_SEED = 7

TORCH_DTYPE = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32, "i32": torch.int32}


def case_seed(base_seed: int, case_index: int) -> int:
    return int(base_seed) + CASE_SEED_STRIDE * (int(case_index) + 1)


def generator(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    return g


def sample(case: str, shape, seed: int, dtype: str, *, mag: float = 1.0, large: float | None = None, spike: float = 100.0) -> torch.Tensor:
    """One adversarial float32 sample (tasks/rmsnorm/reference.py:28-67)."""
    g = generator(seed)
    shape = tuple(int(s) for s in shape)
    dmax = FLOAT_MAX.get(dtype, 3.0e38)
    if case == "normal":
        return torch.randn(shape, generator=g) * mag
    if case == "wide_range":
        e = torch.rand(shape, generator=g) * 5 - 3
        s = torch.where(torch.rand(shape, generator=g) < 0.5, -1.0, 1.0)
        return s * torch.pow(10.0, e) * mag
    if case == "large":
        top = large if large is not None else min(dmax * 0.25, 1.0e4)
        return (torch.rand(shape, generator=g) * 2 - 1) * top
    if case == "tiny":
        if dtype == "fp16":
            lo, hi = TINY_SUBNORMAL["fp16"], TINY_NORMAL["fp16"] * 4
        else:
            lo = TINY_NORMAL.get(dtype, 1.2e-38) * 2.0
            hi = lo * 4096.0
        e = torch.rand(shape, generator=g) * (math.log10(hi) - math.log10(lo)) + math.log10(lo)
        s = torch.where(torch.rand(shape, generator=g) < 0.5, -1.0, 1.0)
        return s * torch.pow(10.0, e)
    if case == "outlier":
        x = torch.randn(shape, generator=g) * mag
        mask = torch.rand(shape, generator=g) < 1e-3
        return torch.where(mask, x * spike, x)
    if case == "cancel":
        x = torch.randn(shape, generator=g) * mag
        big = (torch.rand(shape, generator=g) * 0.5 + 0.5) * 512.0
        s = torch.where(torch.rand(shape, generator=g) < 0.5, -1.0, 1.0)
        v = big * s
        if shape and shape[-1] % 2 == 0:
            vv = v.reshape(*shape[:-1], shape[-1] // 2, 2)
            vv[..., 1] = -vv[..., 0]
            v = vv.reshape(shape)
        return x + v
    if case == "const":
        return torch.full(shape, 1.0 * mag if mag != 1.0 else 0.75)
    raise ValueError(f"unknown case {case!r}")


def inject(t: torch.Tensor, seed: int, max_n: int | None = None) -> torch.Tensor:
    """Plant NaN/+Inf/-Inf/-0.0 (tasks/rmsnorm/reference.py:70-84; first and last element always)."""
    flat = t.reshape(-1).clone()
    numel = flat.numel()
    if numel == 0:
        return flat.reshape(t.shape)
    last = t.shape[-1] if t.dim() else 1
    rows = max(1, numel // max(1, last))
    n = int(min(256, max(8, 0.1 * rows, numel / 65536), max(1, numel // 4)))
    if max_n is not None:
        n = max(2, min(n, max_n))
    perm = torch.randperm(numel, generator=generator(seed))
    perm = perm[(perm != 0) & (perm != numel - 1)]
    pos = torch.cat([torch.tensor([0, numel - 1]), perm[: n - 2]])[:n]
    kinds = torch.randperm(n, generator=generator(seed + 1)) % len(SPECIALS)
    flat[pos] = torch.tensor([SPECIALS[int(k)] for k in kinds], dtype=flat.dtype)
    return flat.reshape(t.shape)


def round_to(t: torch.Tensor, dtype: str) -> torch.Tensor:
    """Round float values to the storage dtype (returned in that dtype)."""
    return t.to(TORCH_DTYPE[dtype])


# ---- per-task streams ------------------------------------------------------------------------

RMSNORM_CASES = ("normal", "wide_range", "large", "tiny", "outlier", "ieee")


def rmsnorm_inputs(case: str, seed: int, rows: int, hidden: int, dtype: str) -> dict[str, torch.Tensor]:
    """tasks/rmsnorm/reference.py:97-107 (mag 1, large 300, w = 1 + 0.1 N(0,1) at seed+99)."""
    base = "normal" if case == "ieee" else case
    x = sample(base, (rows, hidden), seed, dtype, mag=1.0, large=300.0)
    w = 1.0 + 0.1 * sample("normal", (hidden,), seed + 99, dtype)
    if case == "ieee":
        x = inject(x, seed + IEEE_SEED_STRIDE)
        w = inject(w, seed + 2 * IEEE_SEED_STRIDE)
    return {"x": round_to(x, dtype), "w": round_to(w, dtype)}


def rmsnorm_bench_inputs(rows: int, hidden: int, dtype: str, seed: int = SEARCH_SEED) -> dict[str, torch.Tensor]:
    """Timing inputs of the rmsnorm workload: x ~ N(0,1), w ~ U(0.5, 1.5)."""
    g = generator(seed)
    x = torch.randn((rows, hidden), generator=g)
    w = torch.rand((hidden,), generator=g) + 0.5
    return {"x": round_to(x, dtype), "w": round_to(w, dtype)}


GEMM_CASES = ("normal", "wide_range", "large", "tiny", "outlier", "ieee")


def gemm_inputs(case: str, seed: int, a_shape, b_shape, dtype: str) -> dict[str, torch.Tensor]:
    """tasks/gemm/reference.py:86-107: A at seed+0, B at seed+31; mags normal 1 / wide_range
    0.1, large 20, spike 5; the ieee case injects specials into both operands."""
    base = "normal" if case == "ieee" else case
    mag = {"normal": 1.0, "wide_range": 0.1}.get(base, 1.0)
    a = sample(base, a_shape, seed, dtype, mag=mag, large=20.0, spike=5.0)
    b = sample(base, b_shape, seed + 31, dtype, mag=mag, large=20.0, spike=5.0)
    if case == "ieee":
        a = inject(a, seed + IEEE_SEED_STRIDE)
        b = inject(b, seed + 2 * IEEE_SEED_STRIDE)
    return {"A": round_to(a, dtype), "B": round_to(b, dtype)}


def gemm_bench_inputs(m: int, n: int, k: int, dtype: str, seed: int = SEARCH_SEED) -> dict[str, torch.Tensor]:
    """Timing inputs of the dense-gemm workload: A [M,K], B [N,K], both U(-1, 1)."""
    g = generator(seed)
    a = torch.rand((m, k), generator=g) * 2 - 1
    b = torch.rand((n, k), generator=g) * 2 - 1
    return {"A": round_to(a, dtype), "B": round_to(b, dtype)}


# Sampler parameters of the memory-bound tasks: (magnitudes per base case, default magnitude,
# LARGE, SPIKE) from each task's reference.py (softmax :86-89, reduction_sum :86-89,
# silu :86-90, swiglu :86-90, rope :88-91).
MEMBOUND_PARAMS = {
    "softmax": ({"normal": 2.0}, 1.0, 10000.0, 100.0),
    "reduction_sum": ({"normal": 1.0, "wide_range": 0.1}, 1.0, 300.0, 100.0),
    "silu": ({"normal": 3.0}, 1.0, 10000.0, 100.0),
    "swiglu": ({"normal": 3.0}, 1.0, 200.0, 100.0),
    "rope": ({"normal": 1.0, "wide_range": 1.0}, 1.0, 40000.0, 100.0),
    # tasks/relu/reference.py and tasks/sigmoid/reference.py (_MAGS, _DEFAULT_MAG, _LARGE, _SPIKE).
    "relu": ({"normal": 3.0}, 1.0, 10000.0, 100.0),
    "sigmoid": ({"normal": 3.0}, 1.0, 10000.0, 100.0),
    # tasks/sigmoid_shift has no gen_inputs of its own (the harness samples it from the opspec);
    # timing and large-size parity use the sigmoid stream.
    "sigmoid_shift": ({"normal": 3.0}, 1.0, 10000.0, 100.0),
}
MEMBOUND_CASES = {
    "softmax": ("normal", "wide_range", "large", "tiny", "outlier", "const", "ieee"),
    "reduction_sum": ("normal", "wide_range", "large", "tiny", "outlier", "cancel", "ieee"),
    "silu": ("normal", "wide_range", "large", "tiny", "outlier", "ieee"),
    "swiglu": ("normal", "wide_range", "large", "tiny", "outlier", "ieee"),
    "rope": ("normal", "wide_range", "large", "tiny", "outlier", "ieee"),
    "relu": ("normal", "wide_range", "large", "tiny", "outlier", "ieee"),
    "sigmoid": ("normal", "wide_range", "large", "tiny", "outlier", "ieee"),
    "sigmoid_shift": ("normal", "wide_range", "large", "tiny", "outlier", "ieee"),
}
SWIGLU_UP_SEED_STRIDE = 1000003


def membound_inputs(task: str, case: str, seed: int, shape, dtype: str) -> dict[str, torch.Tensor]:
    """Inputs of softmax / reduction_sum / silu / rope (``x``) and swiglu (``gate``, ``up``)."""
    mags, default, large, spike = MEMBOUND_PARAMS[task]
    base = "normal" if case == "ieee" else case
    mag = mags.get(base, default)
    if task == "swiglu":
        gate = sample(base, shape, seed, dtype, mag=mag, large=large, spike=spike)
        up = sample(base, shape, seed + SWIGLU_UP_SEED_STRIDE, dtype, mag=mag, large=large, spike=spike)
        if case == "ieee":
            gate = inject(gate, seed + IEEE_SEED_STRIDE)
            up = inject(up, seed + 2 * IEEE_SEED_STRIDE)
        return {"gate": round_to(gate, dtype), "up": round_to(up, dtype)}
    x = sample(base, shape, seed, dtype, mag=mag, large=large, spike=spike)
    if case == "ieee":
        x = inject(x, seed + IEEE_SEED_STRIDE)
    return {"x": round_to(x, dtype)}


# ---- lion / gemv / gemm_silu ------------------------------------------------------------------

LION_CASES = ("normal", "wide_range", "large", "tiny", "outlier", "ieee")
# tasks/lion/opspec.json attrs defaults.
LION_DEFAULTS = {"LR": 0.001, "WD": 0.1, "BETA1": 0.9, "BETA2": 0.99}


def lion_inputs(case: str, seed: int, n: int, dtype: str) -> dict[str, torch.Tensor]:
    """tasks/lion/reference.py gen_inputs: p, g, m at seed + 7*index (mag 1, large 1000, spike
    100); the tiny case is scaled by 1000 off fp16; ieee injects specials into each of p, g, m at
    seed + 104729*(index+1)."""
    base = "normal" if case == "ieee" else case
    out = {}
    for index, name in enumerate(("p", "g", "m")):
        out[name] = sample(base, (n,), seed + 7 * index, dtype, mag=1.0, large=1000.0)
    if case == "tiny" and dtype != "fp16":
        out = {k: v * 1000.0 for k, v in out.items()}
    if case == "ieee":
        for index, name in enumerate(("p", "g", "m")):
            out[name] = inject(out[name], seed + IEEE_SEED_STRIDE * (index + 1))
    return {k: round_to(v, dtype) for k, v in out.items()}


GEMV_CASES = ("normal", "wide_range", "large", "tiny", "outlier", "ieee")


def gemv_inputs(case: str, seed: int, m: int, k: int, dtype: str) -> dict[str, torch.Tensor]:
    """tasks/gemv/reference.py gen_inputs: A at seed, x at seed + 31 (mags normal 1 / wide_range
    0.1, large 20, spike 5); ieee injects specials into A only."""
    base = "normal" if case == "ieee" else case
    mag = {"normal": 1.0, "wide_range": 0.1}.get(base, 1.0)
    a = sample(base, (m, k), seed, dtype, mag=mag, large=20.0, spike=5.0)
    x = sample(base, (k,), seed + 31, dtype, mag=mag, large=20.0, spike=5.0)
    if case == "ieee":
        a = inject(a, seed + IEEE_SEED_STRIDE)
    return {"A": round_to(a, dtype), "x": round_to(x, dtype)}


# tasks/gemm_silu/reference.py gen_inputs draws A and B exactly like tasks/gemm (same seeds offsets,
# magnitudes, LARGE/SPIKE and ieee injection), so gemm_inputs serves both.
GEMM_SILU_CASES = GEMM_CASES


# ---- kda (fixed length) ------------------------------------------------------------------------

KDA_FIXED_CASES = ("normal", "wide_range", "outlier")


def _kda_fixed_sample(case: str, shape, g: torch.Generator) -> torch.Tensor:
    if case == "normal":
        return torch.randn(shape, generator=g) * 0.5
    if case == "wide_range":
        exponent = torch.rand(shape, generator=g) * 4.0 - 2.0
        sign = torch.where(torch.rand(shape, generator=g) < 0.5, -1.0, 1.0)
        return sign * torch.pow(10.0, exponent) * 0.25
    if case == "outlier":
        values = torch.randn(shape, generator=g) * 0.5
        mask = torch.rand(shape, generator=g) < 0.01
        return torch.where(mask, values * 5.0, values)
    raise ValueError(f"unknown fixed KDA case {case!r}")


def kda_fixed_inputs(case: str, seed: int, n: int, heads: int, dim: int, dtype: str) -> dict[str, torch.Tensor]:
    """tasks/kda/reference.py gen_inputs: one generator at ``seed`` drawn in order A_log =
    log U(1, 16) [H]; dt = exp(U(log 1e-3, log 0.1)) clamped >= 1e-4 [H*D] and dt_bias = dt +
    log(-expm1(-dt)); q, k, v, g [N,H,D] and beta [N,H] from the case sampler; initial_state =
    0.25 N(0,1) [H,D,D] plus 0.5 on the diagonal; scale = 1/sqrt(D).  q..beta rounded to dtype,
    the rest fp32."""
    g = torch.Generator().manual_seed(int(seed))
    a_log = torch.log(torch.empty(heads).uniform_(1.0, 16.0, generator=g))
    dt = torch.exp(
        torch.rand(heads * dim, generator=g) * (torch.log(torch.tensor(0.1)) - torch.log(torch.tensor(0.001)))
        + torch.log(torch.tensor(0.001))
    ).clamp_(min=1e-4)
    dt_bias = dt + torch.log(-torch.expm1(-dt))
    q, k, v, gg = (_kda_fixed_sample(case, (n, heads, dim), g) for _ in range(4))
    beta = _kda_fixed_sample(case, (n, heads), g)
    state0 = torch.randn((heads, dim, dim), generator=g) * 0.25
    state0.diagonal(dim1=-2, dim2=-1).add_(0.5)
    out = {name: round_to(t, dtype) for name, t in (("q", q), ("k", k), ("v", v), ("g", gg), ("beta", beta))}
    out.update({"A_log": a_log.float(), "dt_bias": dt_bias.float(), "initial_state": state0.float(),
                "scale": torch.tensor([1.0 / (dim ** 0.5)], dtype=torch.float32)})
    return out


# ---- bitdelta ---------------------------------------------------------------------------------

BITDELTA_CASES = ("random", "edge_bits", "large", "tiny", "outlier", "ieee")
BITDELTA_EDGE_WORDS = (0, -1, 1431655765, -1431655766, 1, -2147483648, 252645135, -252645136)


def bitdelta_inputs(case: str, seed: int, m: int, n: int, k: int, dtype: str) -> dict[str, torch.Tensor]:
    """tasks/bitdelta_gemm/reference.py:101-124: packed words [K/32, N] (uniform 32-bit, or the
    edge words for ``edge_bits``) from a generator at ``seed``, x at ``seed + 5`` (mag 1, large 20,
    spike 5; edge_bits/random sample x as normal); ieee injects x only."""
    base = "random" if case == "ieee" else case
    g = torch.Generator().manual_seed(int(seed) & 2147483647)
    kb = k // 32
    if base == "edge_bits":
        edge = torch.tensor(BITDELTA_EDGE_WORDS, dtype=torch.int64)
        words = edge[torch.randint(0, len(edge), (kb, n), generator=g)]
    else:
        words = torch.randint(-(1 << 31), 1 << 31, (kb, n), generator=g, dtype=torch.int64)
    xcase = {"edge_bits": "normal", "random": "normal"}.get(base, base)
    x = sample(xcase, (m, k), seed + 5, dtype, mag=1.0, large=20.0, spike=5.0)
    if case == "ieee":
        x = inject(x, seed + IEEE_SEED_STRIDE)
    return {"x": round_to(x, dtype), "bits": words.to(torch.int32)}


BITDELTA_BASE_CASES = ("normal", "large", "ieee")


def bitdelta_base_inputs(case: str, seed: int, m: int, n: int, k: int, dtype: str) -> dict[str, torch.Tensor]:
    """The 1-bit-delta workload: x ~ N(0,1) [M,K], W_base ~ N(0, 0.02) [N,K], S ~ Bernoulli(0.5)
    packed along K into int32 words [N, K/32], alpha ~ U(1e-3, 1e-2) [N].  ``large`` scales x by
    20; ``ieee`` plants specials in x."""
    g = generator(seed)
    x = torch.randn((m, k), generator=g)
    if case == "large":
        x = x * 20.0
    w = torch.randn((n, k), generator=g) * 0.02
    s_bits = torch.randint(0, 2, (n, k // 32, 32), generator=g, dtype=torch.int64)
    shifts = torch.arange(32, dtype=torch.int64)
    words = (s_bits << shifts).sum(-1)
    words = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)
    alpha = torch.rand((n,), generator=g) * (1e-2 - 1e-3) + 1e-3
    if case == "ieee":
        x = inject(x, seed + IEEE_SEED_STRIDE)
    return {"x": round_to(x, dtype), "w_base": round_to(w, dtype), "s_words": words, "alpha": round_to(alpha, dtype)}


# ---- attention --------------------------------------------------------------------------------

ATTENTION_CASES = ("normal", "wide_range", "large", "tiny", "outlier", "ieee")


def attention_inputs(case: str, seed: int, shape, dtype: str) -> dict[str, torch.Tensor]:
    """tasks/flash_attention/reference.py:88-110: q/k/v at seed + 0/31/62 (mags normal 1 /
    wide_range 0.1, large 6, spike 5); the ieee case injects specials into q only."""
    base = "normal" if case == "ieee" else case
    mag = {"normal": 1.0, "wide_range": 0.1}.get(base, 1.0)
    out = {}
    for name, off in (("q", 0), ("k", 31), ("v", 62)):
        out[name] = sample(base, shape, seed + off, dtype, mag=mag, large=6.0, spike=5.0)
    if case == "ieee":
        out["q"] = inject(out["q"], seed + IEEE_SEED_STRIDE)
    return {k: round_to(v, dtype) for k, v in out.items()}


def attention_bench_inputs(shape, dtype: str, seed: int = SEARCH_SEED) -> dict[str, torch.Tensor]:
    """Timing inputs of the causal attention workload: q, k, v ~ N(0, 1)."""
    g = generator(seed)
    return {name: round_to(torch.randn(shape, generator=g), dtype) for name in ("q", "k", "v")}


# ---- varlen KDA -------------------------------------------------------------------------------


def cu_from_lengths(lengths) -> torch.Tensor:
    offs = [0]
    for n in lengths:
        offs.append(offs[-1] + int(n))
    return torch.tensor(offs, dtype=torch.int32)


def kda_gated_lengths(seed: int = SEARCH_SEED, num_seqs: int = 8, lo: int = 256, hi: int = 4096) -> list[int]:
    """The workload's packed sequence lengths: seeded U(lo, hi) integers."""
    g = generator(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (num_seqs,), generator=g)]


def kda_gated_inputs(lengths, heads: int, dim: int, dtype: str, seed: int = SEARCH_SEED, logit_shift: float = 0.0,
                     g_const: float | None = None) -> dict[str, torch.Tensor]:
    """The gated KDA workload: q, k ~ N(0,1) then L2-normalised per head (in fp32, then rounded),
    v ~ N(0,1), beta = sigmoid(N(0,1)) fp32 [T,H], g = logsigmoid(N(0,1) + logit_shift) fp32
    [T,H,D], or g = g_const everywhere when given (strong-decay variants of the workload)."""
    g = generator(seed + 1)
    t = int(sum(lengths))
    q = torch.randn((t, heads, dim), generator=g)
    k = torch.randn((t, heads, dim), generator=g)
    v = torch.randn((t, heads, dim), generator=g)
    q = q / q.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    k = k / k.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    beta = torch.sigmoid(torch.randn((t, heads), generator=g))
    gl = torch.nn.functional.logsigmoid(torch.randn((t, heads, dim), generator=g) + logit_shift)
    if g_const is not None:
        gl = torch.full_like(gl, float(g_const))
    return {"q": round_to(q, dtype), "k": round_to(k, dtype), "v": round_to(v, dtype), "g": gl.float(), "beta": beta.float(),
            "cu_seqlens": cu_from_lengths(lengths)}


def kda_task_inputs(lengths, heads: int, dim: int, dtype: str, seed: int) -> dict[str, torch.Tensor]:
    """Task-contract KDA inputs with the distributions of tasks/varlen_kda/reference.py:420-446
    (0.5 N(0,1) q/k/v/g/beta, A_log = log U(1,16), dt_bias from dt ~ logU(1e-3, 1e-1), a distinct
    non-zero initial state per sequence, scale = 1/sqrt(D))."""
    gen = generator(seed)
    t = int(sum(lengths))
    n = len(lengths)
    rn = lambda shape, s=0.5: torch.randn(shape, generator=gen) * s  # noqa: E731
    a_log = torch.log(torch.empty(heads).uniform_(1.0, 16.0, generator=gen))
    lo, hi = math.log(0.001), math.log(0.1)
    dt = torch.exp(torch.rand(heads * dim, generator=gen) * (hi - lo) + lo).clamp_(min=1e-4)
    dt_bias = dt + torch.log(-torch.expm1(-dt))
    q, k, v, gg = (rn((t, heads, dim)) for _ in range(4))
    beta = rn((t, heads))
    s0 = rn((n, heads, dim, dim), 0.25)
    for s in range(n):
        s0[s].diagonal(dim1=-2, dim2=-1).add_(0.5 + 0.25 * s)
    return {
        "q": round_to(q, dtype), "k": round_to(k, dtype), "v": round_to(v, dtype), "g": round_to(gg, dtype),
        "beta": round_to(beta, dtype), "A_log": a_log.float(), "dt_bias": dt_bias.float(), "initial_state": s0.float(),
        "cu_seqlens": cu_from_lengths(lengths), "scale": torch.tensor([1.0 / math.sqrt(dim)], dtype=torch.float32),
    }


# ---- mamba2 chunk scan ------------------------------------------------------------------------

MAMBA2_CASES = ("normal", "wide_range", "large", "tiny", "outlier", "ieee")
MAMBA2_OFFSETS = {"x": 0, "Bmat": 31, "Cmat": 62, "states": 93, "Dskip": 124, "dt": 155, "decay": 186}


def mamba2_inputs(case: str, seed: int, batch: int, seq: int, heads: int, headdim: int, dstate: int, chunk: int,
                  dtype: str) -> dict[str, torch.Tensor]:
    """tasks/mamba2_chunk_scan/reference.py:199-223: dt = round(0.001 + 0.049 sigmoid(N(0,1))),
    A = -(1 + 7 sigmoid(N(0,1))) per head, dA_cumsum = the in-chunk cumulative sum of dt*A laid out
    [B,H,NC,CHUNK]; x/B/C/D/states from the case sampler (mags normal 1 / wide_range 0.1, large 4,
    spike 5); the ieee case injects specials into states only."""
    base = "normal" if case == "ieee" else case
    mag = {"normal": 1.0, "wide_range": 0.1}.get(base, 1.0)
    nc = seq // chunk
    off = MAMBA2_OFFSETS
    dt = round_to(0.001 + 0.049 * torch.sigmoid(sample("normal", (batch, seq, heads), seed + off["dt"], dtype)), dtype).float()
    a = -(1.0 + 7.0 * torch.sigmoid(sample("normal", (heads,), seed + off["decay"], dtype)))
    cs = (dt.reshape(batch, nc, chunk, heads) * a).cumsum(dim=2).permute(0, 3, 1, 2).contiguous()
    kw = dict(mag=mag, large=4.0, spike=5.0)
    out = {
        "x": sample(base, (batch, seq, heads, headdim), seed + off["x"], dtype, **kw),
        "dt": dt,
        "dA_cumsum": cs,
        "Bmat": sample(base, (batch, seq, dstate), seed + off["Bmat"], dtype, **kw),
        "Cmat": sample(base, (batch, seq, dstate), seed + off["Cmat"], dtype, **kw),
        "Dskip": sample(base, (heads,), seed + off["Dskip"], dtype, **kw),
        "states": sample(base, (batch, nc, heads, headdim, dstate), seed + off["states"], dtype, **kw),
    }
    if case == "ieee":
        out["states"] = inject(out["states"], seed + 7 * IEEE_SEED_STRIDE)
    return {k: round_to(v, dtype) for k, v in out.items()}
