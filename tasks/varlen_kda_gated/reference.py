"""varlen_kda_gated: the gated delta rule over packed variable-length sequences -- the gated KDA
workload, a variant of tasks/varlen_kda (which normalises q/k in-op, derives the log-decay from
A_log / dt_bias / LOWER_BOUND, sigmoids beta and starts from a given state).

Per sequence s and head h, with an fp64 state S [D_v, D_k] starting at zero:
    S <- S diag(exp(g_t));  r = beta_t (v_t - S k_t);  S <- S + r k_t^T;  o_t = S (q_t / sqrt(D)).
q and k arrive L2-normalised, g is the per-channel log-decay used as given and beta the gate
used as given.  Values: q, k, v ~ N(0,1) with q, k normalised per token and head,
beta = sigmoid(N(0,1)), g = logsigmoid(N(0,1)) (the workload distribution); strong_decay shifts
the decay logits by -3, decay_shift8 by -8, constant_decay6 sets every log-decay to -6,
extreme_decay draws them around -30 with a few exact zeros of the decay (g = -inf), and wide_v
scales v by 100.  The decay cases span the range a chunked kernel has to survive: cumulative
log-decays of -100 to -500 over 16 tokens, and infinite ones.

Segmentation: every case keeps the tier's total token count and sequence count (the packed
shapes are fixed) and re-cuts the batch: canonical (the declared lengths), permuted, skewed (one
long sequence, the rest of length 1), all_unaligned_primes (prime lengths, the last one takes the
remainder), max_handoff_stress (lengths 16k +- 1 so sequences straddle 16-token chunk edges),
chunk_boundary (multiples of 16), zero_length (every other sequence empty), single_sequence (one
sequence holds every token) and fresh_distribution (seeded random cut points).  The decay cases and
wide_v use the canonical cut.
"""

import math

import torch


def _generator(seed):
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed) & 0x7FFFFFFFFFFFFFFF)
    return g


def _offsets(lengths):
    offs = [0]
    for n in lengths:
        offs.append(offs[-1] + int(n))
    return offs


def _is_prime(n):
    if n < 2:
        return False
    f = 2
    while f * f <= n:
        if n % f == 0:
            return False
        f += 1
    return True


def _fit(lengths, total):
    """Make the lengths sum to `total` by changing the last one (kept >= 0), else spread evenly."""
    rest = total - sum(lengths[:-1])
    if rest >= 0:
        return lengths[:-1] + [rest]
    n = len(lengths)
    return [total // n + (1 if i < total % n else 0) for i in range(n)]


def _cut(case, canonical, seed):
    n, total = len(canonical), sum(canonical)
    g = _generator(seed + 4099)
    if case in ("canonical", "wide_v") or case in DECAY_CASES:
        return list(canonical)
    if case == "permuted":
        return [canonical[i] for i in torch.randperm(n, generator=g).tolist()]
    if case == "skewed":
        return [total] if n == 1 else _fit([total - (n - 1)] + [1] * (n - 1), total)
    if case == "all_unaligned_primes":
        base = max(3, total // n)
        primes = []
        for i in range(n - 1):
            c = max(3, base - 7 * i)
            while not _is_prime(c):
                c -= 1
            primes.append(max(c, 2))
        return _fit(primes + [0], total)
    if case == "max_handoff_stress":
        unit = max(1, total // (16 * n))
        return _fit([max(1, 16 * unit + (1 if i % 2 == 0 else -1)) for i in range(n)], total)
    if case == "chunk_boundary":
        return _fit([16 * max(1, (total // n) // 16) for _ in range(n)], total)
    if case == "zero_length":
        live = [i for i in range(n) if i % 2 == 1] or [0]
        out = [0] * n
        for j, i in enumerate(live):
            out[i] = total // len(live) + (1 if j < total % len(live) else 0)
        return out
    if case == "single_sequence":
        return [total] + [0] * (n - 1)
    if case == "fresh_distribution":
        cuts = sorted(torch.randint(0, total + 1, (n - 1,), generator=g).tolist())
        edges = [0] + cuts + [total]
        return [edges[i + 1] - edges[i] for i in range(n)]
    raise ValueError(f"unknown case {case!r}")


DECAY_CASES = ("strong_decay", "decay_shift8", "constant_decay6", "extreme_decay")


def gen_inputs(case, seed, instance):
    lengths = _cut(case, [int(x) for x in instance.canonical_seq_lens], seed)
    heads, dim = int(instance.symbols["H"]), int(instance.symbols["D"])
    total = sum(lengths)
    g = _generator(seed)
    f64 = torch.float64
    q = torch.randn((total, heads, dim), generator=g, dtype=f64)
    k = torch.randn((total, heads, dim), generator=g, dtype=f64)
    v = torch.randn((total, heads, dim), generator=g, dtype=f64)
    q = q / q.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    k = k / k.norm(dim=-1, keepdim=True).clamp_min(1e-12)
    beta = torch.sigmoid(torch.randn((total, heads), generator=g, dtype=f64))
    logits = torch.randn((total, heads, dim), generator=g, dtype=f64)
    if case == "strong_decay":
        logits = logits - 3.0
    elif case == "decay_shift8":
        logits = logits - 8.0
    elif case == "wide_v":
        v = v * 100.0
    decay = torch.nn.functional.logsigmoid(logits)
    if case == "constant_decay6":
        decay = torch.full_like(decay, -6.0)
    elif case == "extreme_decay":
        decay = -30.0 + 5.0 * torch.randn(decay.shape, generator=g, dtype=f64)
        zero = torch.rand(decay.shape, generator=g, dtype=f64) < 0.01
        decay = torch.where(zero, torch.full_like(decay, -math.inf), decay)
    return {"q": q, "k": k, "v": v, "g": decay, "beta": beta,
            "cu_seqlens": torch.tensor(_offsets(lengths), dtype=torch.int32)}


def reference(inputs, attrs):
    q, k, v, g = (inputs[n].double() for n in ("q", "k", "v", "g"))
    beta = inputs["beta"].double()
    cu = [int(x) for x in inputs["cu_seqlens"].tolist()]
    total, heads, dim = q.shape
    scale = 1.0 / math.sqrt(dim)
    out = torch.zeros((total, heads, dim), dtype=torch.float64)
    final = torch.zeros((len(cu) - 1, heads, dim, dim), dtype=torch.float64)
    for s in range(len(cu) - 1):
        state = torch.zeros((heads, dim, dim), dtype=torch.float64)
        for t in range(cu[s], cu[s + 1]):
            state = state * torch.exp(g[t]).unsqueeze(1)
            r = (v[t] - torch.einsum("hvk,hk->hv", state, k[t])) * beta[t].unsqueeze(-1)
            state = state + r.unsqueeze(-1) * k[t].unsqueeze(1)
            out[t] = torch.einsum("hvk,hk->hv", state, q[t] * scale)
        final[s] = state
    return {"output": out, "final_state": final}
