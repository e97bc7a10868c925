"""bitdelta_gemm_base: y = x . (W_base + diag(alpha) S)^T -- the 1-bit-delta workload, a variant
of tasks/bitdelta_gemm (which has no base weight, a scalar scale and signs packed [K/32, N]).

S[n, k] = +1 when bit (k % 32) of s_words[n, k // 32] is set, else -1 (signs packed along K, one
row of words per output column n).  Oracle in fp64, as the two products the workload is defined
by, y = x . W_base^T + alpha * (x . S^T) (equal to the merged form for finite inputs; with a
non-finite x element the two products fix which NaN / +-Inf results).  Cases: normal (x ~ N(0,1), W_base ~
N(0, 0.02), alpha ~ U(1e-3, 1e-2), Bernoulli(0.5) signs -- the workload distribution), large
(x ~ U(-4,4), W_base ~ U(-1,1)), edge_bits (whole words of fixed patterns: all set, none set,
alternating, nibble blocks) and ieee (normal with NaN/+-Inf/-0 placed in x).
"""

import torch

_SPECIALS = (float("nan"), float("inf"), float("-inf"), -0.0)
_EDGE_WORDS = (0, -1, 0x55555555, -0x55555556, 1, -(1 << 31), 0x0F0F0F0F, -0x0F0F0F10)


def _generator(seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    return g


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
    kw = k // 32
    f64 = torch.float64
    gx, gw, gs, ga = (_generator(seed + off) for off in (0, 31, 62, 93))
    if case == "large":
        x = (torch.rand((m, k), generator=gx, dtype=f64) * 2.0 - 1.0) * 4.0
        w = torch.rand((n, k), generator=gw, dtype=f64) * 2.0 - 1.0
    else:
        x = torch.randn((m, k), generator=gx, dtype=f64)
        w = torch.randn((n, k), generator=gw, dtype=f64) * 0.02
    if case == "edge_bits":
        pick = torch.randint(0, len(_EDGE_WORDS), (n, kw), generator=gs)
        words = torch.tensor(_EDGE_WORDS, dtype=torch.int64)[pick]
    else:
        words = torch.randint(-(1 << 31), 1 << 31, (n, kw), generator=gs, dtype=torch.int64)
    alpha = torch.rand((n,), generator=ga, dtype=f64) * 9e-3 + 1e-3
    if case == "ieee":
        x = _place_specials(x, seed + 7)
    return {"x": x, "w_base": w, "s_words": words, "alpha": alpha}


def _signs(words, k):
    """[N, K/32] words -> [N, K] of +-1 (bit j of word kb is column kb*32 + j)."""
    w = words.to(torch.int64) & 0xFFFFFFFF
    bits = (w.unsqueeze(-1) >> torch.arange(32, dtype=torch.int64)) & 1
    return (bits.reshape(w.shape[0], -1)[:, :k] * 2 - 1).to(torch.float64)


def reference(inputs, attrs):
    x = inputs["x"].double()
    w = inputs["w_base"].double()
    s = _signs(inputs["s_words"], w.shape[1])
    return {"y": x @ w.transpose(0, 1) + inputs["alpha"].double().reshape(1, -1) * (x @ s.transpose(0, 1))}
