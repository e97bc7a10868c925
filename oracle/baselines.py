"""The reference's registered timing baselines, restated as torch calls on CPU tensors.

TEST AND MEASUREMENT INFRASTRUCTURE ONLY, like the rest of this package: ``bench.py`` times these
on the host cores beside the GPU numbers.  Each task's ``baselines.py`` registers library calls
(``torch_mps``: plain torch) that the harness times a candidate against; the B200 box has no MPS
device and the reference tree does not travel there, so the same calls run here on CPU tensors,
in the task's storage dtype.  The workload variants get the same call on their layout.

``registered(name, inputs, sample)`` returns ``(callable, algorithmic units of one call,
description)`` for a bounded sample of the workload (rows of A, heads of attention, one KDA chain),
so that a timing stays within seconds.
"""

from __future__ import annotations

import math

import torch


def rmsnorm(x, w, eps=1e-6):
    """tasks/rmsnorm/baselines.py torch_mps: ``F.rms_norm(x, (H,), w, eps)``."""
    return torch.nn.functional.rms_norm(x, (x.shape[-1],), w, eps)


def gemm_nt(a, b):
    """tasks/gemm/baselines.py torch_mps (``torch.matmul``) on the C = A.B^T layout."""
    return torch.matmul(a, b.t())


def bitdelta_gemm_base(x, w_base, s_words, alpha):
    """The bitdelta baseline's torch decode (tasks/bitdelta_gemm/baselines.py ``_torch_decode``:
    bit j of a word is element 32*word + j, set = +1) on the workload's [N, K/32] packing, then
    one dense matmul ``x @ (W_base + diag(alpha) S)^T``."""
    n, kw = s_words.shape
    j = torch.arange(32, dtype=torch.int32).reshape(1, 1, 32)
    bits = (s_words.to(torch.int32).reshape(n, kw, 1) >> j) & 1
    s = (bits.to(x.dtype) * 2 - 1).reshape(n, kw * 32)
    return x @ (w_base + alpha[:, None] * s).t()


def attention(q, k, v, causal=True):
    """tasks/flash_attention/baselines.py torch_mps: ``F.scaled_dot_product_attention`` (with the
    causal mask for the causal configuration, scale 1/sqrt(D))."""
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal, scale=1.0 / math.sqrt(q.shape[-1]))


def kda_gated(q, k, v, g, beta, cu_seqlens, scale):
    """tasks/varlen_kda/baselines.py ``run``: the token-by-token delta rule in fp32 torch, with the
    gated workload's supplied log-decay and gate (q/k already normalised, state from zero)."""
    q, k, v, g, beta = (t.to(torch.float32) for t in (q, k, v, g, beta))
    cu = [int(c) for c in cu_seqlens]
    heads, dim = q.shape[1], q.shape[2]
    out = torch.zeros_like(v)
    final = torch.zeros((len(cu) - 1, heads, v.shape[2], dim))
    for s in range(len(cu) - 1):
        state = torch.zeros((heads, v.shape[2], dim))
        for t in range(cu[s], cu[s + 1]):
            state = state * torch.exp(g[t])[:, None, :]
            r = (v[t] - (state * k[t][:, None, :]).sum(-1)) * beta[t][:, None]
            state = state + r[:, :, None] * k[t][:, None, :]
            out[t] = (state * (q[t] * scale)[:, None, :]).sum(-1)
        final[s] = state
    return out, final


def registered(name: str, inputs: dict, sample: int):
    """The registered baseline of workload ``name`` on a sample of ``inputs`` (CPU tensors)."""
    if name.startswith("rmsnorm"):
        x, w = inputs["x"][:sample], inputs["w"]
        r, h = x.shape
        return (lambda: rmsnorm(x, w)), 4.0 * r * h + 2.0 * h, f"F.rms_norm on {r} of the rows ({x.dtype})"
    if name.startswith("gemm_nt"):
        a, b = inputs["A"][:sample], inputs["B"]
        return (lambda: gemm_nt(a, b)), 2.0 * a.shape[0] * b.shape[0] * a.shape[1], f"torch.matmul(A, B^T) on {a.shape[0]} rows of A ({a.dtype})"
    if name.startswith("bitdelta_base"):
        x, w, s, al = inputs["x"], inputs["w_base"][:sample], inputs["s_words"][:sample], inputs["alpha"][:sample]
        m, kk = x.shape
        n = w.shape[0]
        nbytes = 2.0 * n * kk + n * kk / 8 + 2.0 * n + 2.0 * m * kk + 2.0 * m * n
        return (lambda: bitdelta_gemm_base(x, w, s, al)), nbytes, f"torch sign decode + matmul over {n} output columns ({x.dtype})"
    if name.startswith("attention"):
        b, h, s_len, d = inputs["q"].shape
        flat = [inputs[n_].reshape(b * h, s_len, d)[:sample].unsqueeze(0) for n_ in ("q", "k", "v")]
        causal = "causal" in name
        fl = 4.0 * sample * d * (s_len * (s_len + 1) / 2 if causal else s_len * s_len)
        return (lambda: attention(*flat, causal=causal)), fl, f"F.scaled_dot_product_attention on {sample} of the {b * h} heads ({flat[0].dtype})"
    if name.startswith("kda_gated"):
        t = min(sample, int(inputs["cu_seqlens"][1]))
        sl = {n_: inputs[n_][:t, :1] for n_ in ("q", "k", "v", "g", "beta")}
        dim = sl["q"].shape[-1]
        per_token = 3 * 2 * dim + 4 * dim + 4 + 2 * dim
        return ((lambda: kda_gated(sl["q"], sl["k"], sl["v"], sl["g"], sl["beta"], [0, t], 1.0 / math.sqrt(dim))),
                float(per_token * t), f"token-by-token torch delta rule over {t} tokens of one chain")
    raise KeyError(name)
