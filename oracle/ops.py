"""fp64 numpy restatements of the task operators (test infrastructure only).

Every function takes float64 arrays (already widened from the storage dtype) and returns
float64 results, like the reference's ``reference(inputs, attrs)`` functions, which widen the
rounded inputs and apply the formula once in fp64.
"""

from __future__ import annotations

import numpy as np

def _err():
    return np.errstate(all="ignore")


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """tasks/rmsnorm/reference.py:110-115: ``x * rsqrt(mean(x*x, -1) + eps) * w``."""
    with _err():
        ms = np.mean(x * x, axis=-1, keepdims=True)
        return x * (1.0 / np.sqrt(ms + eps)) * w


def softmax(x: np.ndarray) -> np.ndarray:
    """tasks/softmax/reference.py:104-106: row softmax over the last axis (torch.softmax rules:
    the row max is subtracted first; a NaN or +Inf in a row makes the row NaN, -Inf entries
    get weight 0, an all -Inf row is NaN)."""
    with _err():
        m = np.max(x, axis=-1, keepdims=True)
        nan_row = np.isnan(x).any(axis=-1, keepdims=True)
        e = np.exp(x - m)
        y = e / np.sum(e, axis=-1, keepdims=True)
        return np.where(nan_row, np.nan, y)


def reduction_sum(x: np.ndarray) -> np.ndarray:
    """tasks/reduction_sum/reference.py:104-106: row sum in fp64."""
    with _err():
        return np.sum(x, axis=-1)


def reduction_sum_error_scale(x: np.ndarray) -> np.ndarray:
    """tasks/reduction_sum/reference.py:109-113: per-row ``sum |x|`` over the finite inputs."""
    fin = np.where(np.isfinite(x), x, 0.0)
    return np.sum(np.abs(fin), axis=-1)


def _sigmoid(x):
    with _err():
        return np.where(x >= 0, 1.0 / (1.0 + np.exp(-x)), np.exp(x) / (1.0 + np.exp(x)))


def silu(x: np.ndarray) -> np.ndarray:
    """tasks/silu/reference.py:105-108: ``x * sigmoid(x)``."""
    with _err():
        return x * _torch_sigmoid(x)


def _torch_sigmoid(x):
    # torch.sigmoid(x) in fp64 is 1 / (1 + exp(-x)); keep that exact form so +-Inf and NaN map
    # the way the reference's fp64 tensors do (sigmoid(-inf) = 0, sigmoid(inf) = 1).
    with _err():
        return 1.0 / (1.0 + np.exp(-x))


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """tasks/swiglu/reference.py:109-113: ``gate * sigmoid(gate) * up``."""
    with _err():
        return gate * _torch_sigmoid(gate) * up


def relu(x: np.ndarray) -> np.ndarray:
    """tasks/relu/reference.py ``reference``: ``torch.relu`` in fp64 (x > 0 keeps x, NaN stays
    NaN, everything else is +0)."""
    return np.where(np.isnan(x), x, np.where(x > 0, x, 0.0))


def sigmoid(x: np.ndarray) -> np.ndarray:
    """tasks/sigmoid/reference.py ``reference``: ``torch.sigmoid`` in fp64."""
    return _torch_sigmoid(x)


def sigmoid_shift(x: np.ndarray) -> np.ndarray:
    """tasks/sigmoid_shift/reference.py ``reference``: ``sigmoid(x) + 1`` in fp64 (the module then
    stores fp32; the harness rounds that to the output dtype)."""
    with _err():
        return (_torch_sigmoid(x) + 1.0).astype(np.float32).astype(np.float64)


def lion(p: np.ndarray, g: np.ndarray, m: np.ndarray, lr: float, wd: float, beta1: float, beta2: float):
    """tasks/lion/reference.py ``reference``: one fp64 Lion step; returns ``(p_out, m_out)``.
    ``torch.sign`` maps NaN to 0 (numpy's sign keeps NaN), so a NaN ``c`` leaves ``p`` decayed only."""
    with _err():
        c = beta1 * m + (1 - beta1) * g
        u = np.where(np.isnan(c), 0.0, np.sign(c))
        return p * (1 - lr * wd) - lr * u, beta2 * m + (1 - beta2) * g


# tasks/lion/reference.py module constants of the sign-discontinuity allowance.
LION_DISCONTINUITY_REL = 1e-05
LION_ATOL_STEPS = 2.5


def lion_error_scale(p, g, m, p_out_ref, m_out_ref, lr: float, beta1: float, atol_rel: float):
    """tasks/lion/reference.py ``error_scale``: non-finite inputs/outputs count as 0; ``p_out``'s
    scale is the RMS of its reference, except where ``|a + b| <= 1e-5 (|a| + |b|)``
    (a = beta1*m, b = (1-beta1)*g: the sign of c is ambiguous at fp32 precision), where it is
    ``2.5 * lr / atol_rel`` (2.5 learning-rate steps of slack); ``m_out``'s is its RMS."""
    fin = lambda t: np.where(np.isfinite(t), t, 0.0)  # noqa: E731
    p, g, m = fin(p), fin(g), fin(m)
    rp, rm = fin(p_out_ref), fin(m_out_ref)
    with _err():
        a, b = beta1 * m, (1 - beta1) * g
        amb = np.abs(a + b) <= LION_DISCONTINUITY_REL * (np.abs(a) + np.abs(b))
    base = np.full(rp.shape, np.sqrt(np.mean(rp**2)) if rp.size else 0.0)
    base[amb] = LION_ATOL_STEPS * lr / atol_rel
    return base, np.float64(np.sqrt(np.mean(rm**2)) if rm.size else 0.0)


def gemv(a: np.ndarray, x: np.ndarray) -> np.ndarray:
    """tasks/gemv/reference.py ``reference``: ``A @ x`` in fp64."""
    with _err():
        return a @ x


def gemm_silu(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """tasks/gemm_silu/reference.py ``reference``: ``c = A @ B`` (the reference forms it in fp32;
    the fp64 product here agrees to fp32 accumulation error), then ``c * sigmoid(c)`` in fp64."""
    with _err():
        c = a @ b
        return c * _torch_sigmoid(c)


def rope(x: np.ndarray, base: float) -> np.ndarray:
    """tasks/rope/reference.py:105-115: rotate-half RoPE over ``[..., S, D]``; the position is
    the index along S and ``inv_freq = base ** (-arange(D/2) / (D/2))``."""
    half = x.shape[-1] // 2
    seq = x.shape[-2]
    inv_freq = base ** (-np.arange(half, dtype=np.float64) / half)
    ang = np.arange(seq, dtype=np.float64)[:, None] * inv_freq[None, :]
    c, s = np.cos(ang), np.sin(ang)
    x1, x2 = x[..., :half], x[..., half:]
    with _err():
        return np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1)


def gemm_nn(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """tasks/gemm/reference.py:110-114: ``C = A @ B`` with B ``[K, N]`` (computed in fp64; the
    reference's fp32 product widened to fp64 agrees to fp32 accumulation error)."""
    with _err():
        return a @ b


def gemm_nt(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """``C = A @ B^T`` with B ``[N, K]``: the pinned NN product applied to ``B^T``."""
    return gemm_nn(a, b.T)


def unpack_pm1_kn(words: np.ndarray) -> np.ndarray:
    """tasks/bitdelta_gemm/reference.py:108-116: ``[KB, N]`` 32-bit words -> ``[K, N]`` of +-1,
    bit j of ``words[kb, n]`` is row ``kb*32 + j`` (+1 when set)."""
    w = np.asarray(words).astype(np.int64) & 0xFFFFFFFF
    j = np.arange(32, dtype=np.int64).reshape(1, 32, 1)
    bit = (w[:, None, :] >> j) & 1
    return (bit.astype(np.float64) * 2 - 1).reshape(-1, w.shape[-1])


def bitdelta_gemm(x: np.ndarray, bits: np.ndarray, scale: float) -> np.ndarray:
    """tasks/bitdelta_gemm/reference.py:127-130: ``y = SCALE * (x @ W)``, W = unpack(bits)."""
    with _err():
        return (x @ unpack_pm1_kn(bits)) * scale


def unpack_pm1_nk(words: np.ndarray) -> np.ndarray:
    """``[N, K/32]`` words packed along K -> ``[N, K]`` of +-1 (bit j of ``words[n, kb]`` is
    column ``kb*32 + j``), the same bit order as :func:`unpack_pm1_kn` transposed."""
    return unpack_pm1_kn(np.asarray(words).T).T


def bitdelta_gemm_base(x: np.ndarray, w_base: np.ndarray, s_words: np.ndarray, alpha: np.ndarray) -> np.ndarray:
    """``y = x @ (W_base + diag(alpha) S)^T = x @ W_base^T + alpha * (x @ S^T)`` with S in
    {-1,+1} packed ``[N, K/32]`` along K; alpha scales output column n."""
    s = unpack_pm1_nk(s_words)
    with _err():
        return x @ w_base.T + (x @ s.T) * alpha[None, :]


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, causal: bool = False) -> np.ndarray:
    """tasks/flash_attention/reference.py:113-119: ``softmax(q k^T * scale [+ causal mask]) v``
    over ``[B, H, S, D]`` (scaled_dot_product_attention semantics; the causal mask keeps key
    j <= query i)."""
    with _err():
        s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
        if causal:
            sq, sk = s.shape[-2], s.shape[-1]
            mask = np.tril(np.ones((sq, sk), dtype=bool))
            s = np.where(mask, s, -np.inf)
        p = softmax(s)
        return np.einsum("bhqk,bhkd->bhqd", p, v)


def _sigmoid_t(x):
    with _err():
        return 1.0 / (1.0 + np.exp(-x))


def delta_rule(q: np.ndarray, k: np.ndarray, v: np.ndarray, log_decay: np.ndarray, beta: np.ndarray,
               state0: np.ndarray, cu_seqlens: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The per-token gated delta-rule core of tasks/varlen_kda/reference.py:352-368.

    Inputs are already prepared: ``q``/``k`` ``[T, H, D]`` (normalised; q carries the scale),
    ``log_decay`` ``[T, H, Dk]``, ``beta`` ``[T, H]`` (already sigmoided), ``state0``
    ``[N, H, Dv, Dk]`` (V-first).  Per sequence s and token t:
    ``S *= exp(ld_t)`` along the key axis; ``r = (v_t - S k_t) * beta_t``; ``S += r (x) k_t``;
    ``o_t = S q_t``.  Returns ``(output [T, H, Dv], final_state [N, H, Dv, Dk])``.
    """
    state = np.array(state0, dtype=np.float64, copy=True)
    out = np.zeros(v.shape, dtype=np.float64)
    cu = [int(c) for c in cu_seqlens]
    with _err():
        for s in range(len(cu) - 1):
            st = state[s]
            for t in range(cu[s], cu[s + 1]):
                st = st * np.exp(log_decay[t])[:, None, :]
                r = v[t] - np.einsum("hvk,hk->hv", st, k[t])
                r = r * beta[t][:, None]
                st = st + r[:, :, None] * k[t][:, None, :]
                out[t] = np.einsum("hvk,hk->hv", st, q[t])
            state[s] = st
    return out, state


def varlen_kda(q, k, v, g, beta, a_log, dt_bias, initial_state, cu_seqlens, scale, lower_bound):
    """tasks/varlen_kda/reference.py:323-374: q/k L2 normalisation (``rsqrt(sum x^2 + 1e-6)``,
    q times ``scale``), log-decay ``LOWER_BOUND * sigmoid(exp(A_log) * (g + dt_bias))``,
    ``sigmoid(beta)``, then :func:`delta_rule` per sequence from ``initial_state``."""
    heads, dim = q.shape[1], q.shape[2]
    with _err():
        qn = q / np.sqrt(np.sum(q * q, axis=-1, keepdims=True) + 1e-6) * float(scale)
        kn = k / np.sqrt(np.sum(k * k, axis=-1, keepdims=True) + 1e-6)
        gate = g + np.asarray(dt_bias).reshape(heads, dim)[None]
        ld = float(lower_bound) * _sigmoid_t(np.exp(np.asarray(a_log))[None, :, None] * gate)
        b = _sigmoid_t(beta)
    return delta_rule(qn, kn, v, ld, b, initial_state, cu_seqlens)


def kda_fixed(q, k, v, g, beta, a_log, dt_bias, initial_state, scale, lower_bound):
    """tasks/kda/reference.py ``reference``: the same per-token recurrence as :func:`varlen_kda`
    (normalisation, gated decay, delta residual, V-first state) over one sequence of all N tokens
    from ``initial_state [H, D, D]``; returns ``(output [N,H,D], final_state [H,D,D])``."""
    n = q.shape[0]
    out, fin = varlen_kda(q, k, v, g, beta, a_log, dt_bias, np.asarray(initial_state)[None], np.array([0, n]), scale, lower_bound)
    return out, fin[0]


def varlen_kda_gated(q, k, v, g, beta, cu_seqlens, scale, state0=None):
    """Gated variant: q/k already L2-normalised, ``g`` is the fp32 per-channel log-decay used
    directly, ``beta`` is already sigmoided, the initial state is zero unless given; q is
    multiplied by ``scale`` (1/sqrt(D)) as in the task op."""
    n = len(cu_seqlens) - 1
    heads, dim = q.shape[1], q.shape[2]
    if state0 is None:
        state0 = np.zeros((n, heads, v.shape[2], dim), dtype=np.float64)
    return delta_rule(q * float(scale), k, v, g, beta, state0, cu_seqlens)


def attention_rows(q, k, v, scale: float, causal: bool, rows) -> np.ndarray:
    """:func:`attention` for the query rows ``rows`` only (``[B, H, len(rows), D]``); each output
    row depends only on its own query row, so this equals ``attention(...)[:, :, rows]``."""
    rows = np.asarray(rows)
    with _err():
        s = np.einsum("bhqd,bhkd->bhqk", q[:, :, rows], k) * scale
        if causal:
            keys = np.arange(k.shape[2])
            s = np.where(keys[None, :] <= rows[:, None], s, -np.inf)
        p = softmax(s)
        return np.einsum("bhqk,bhkd->bhqd", p, v)


def mamba2_chunk_scan(x, dt, dA_cumsum, b_mat, c_mat, d_skip, states):
    """tasks/mamba2_chunk_scan/reference.py:106-127 (the Mamba-2 SSD chunk scan, paper listing 1,
    one B/C group), in fp64.  Per batch b, chunk c (rows t = c*CHUNK + l), head h:

        w[l, s]  = (C[t_l] . B[t_s]) * exp(cs[b,h,c,l] - cs[b,h,c,s]) * dt[b,t_s,h]   if s <= l else 0
        y[t_l,h] = sum_s w[l, s] x[t_s, h]
                 + exp(cs[b,h,c,l]) * sum_n C[t_l, n] states[b,c,h,:,n]  +  D[h] x[t_l, h]

    Shapes: x [B,L,H,P], dt [B,L,H], dA_cumsum [B,H,NC,CHUNK], b_mat/c_mat [B,L,N], d_skip [H],
    states [B,NC,H,P,N]; y [B,L,H,P].  Masked entries are exactly zero (``where``) and still multiply
    x, so a non-finite x element makes every row of its chunk non-finite, as in the reference.
    """
    bsz, seq, heads, hd = x.shape
    nc, chunk = dA_cumsum.shape[2], dA_cumsum.shape[3]
    if nc * chunk != seq:
        raise ValueError(f"SEQLEN {seq} != NCHUNKS {nc} * CHUNK {chunk}")
    x5 = np.asarray(x, np.float64).reshape(bsz, nc, chunk, heads, hd)
    dt4 = np.asarray(dt, np.float64).reshape(bsz, nc, chunk, heads).transpose(0, 3, 1, 2)  # [B,H,NC,C]
    cs = np.asarray(dA_cumsum, np.float64)
    br = np.asarray(b_mat, np.float64).reshape(bsz, nc, chunk, -1)
    cr = np.asarray(c_mat, np.float64).reshape(bsz, nc, chunk, -1)
    st = np.asarray(states, np.float64)
    causal = np.tril(np.ones((chunk, chunk), dtype=bool))
    with _err():
        cb = np.einsum("bcln,bcsn->bcls", cr, br)
        decay = np.exp(cs[..., :, None] - cs[..., None, :])                      # [B,H,NC,l,s]
        w = np.where(causal, cb[:, None] * decay * dt4[..., None, :], 0.0)
        y = np.einsum("bhcls,bcshp->bclhp", w, x5)
        y = y + np.einsum("bcln,bchpn->bclhp", cr, st) * np.exp(cs).transpose(0, 2, 3, 1)[..., None]
        y = y + np.asarray(d_skip, np.float64)[:, None] * x5
    return y.reshape(bsz, seq, heads, hd)
