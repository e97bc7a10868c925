"""Naive CUDA fallback providers: one registered implementation per task for shape portfolios.

A shape portfolio (``portfolio_pack``) dispatches each shape to exactly one candidate variant or
to its declared fallback (tcenv/portfolio/candidate.py: fallback kind ``registered_implementation``
with an ``implementation_id`` and ``implementation_version``).  These are the B200 backend's
fallbacks: straightforward, always-correct kernels for every shape of a task, so a portfolio's
``effective_end_to_end`` account times a real kernel where no variant applies.

Each provider renders a single-source cuda-single candidate:

* kernel arguments are the task's ABI tensors in opspec order, then the task's symbols as
  ``long long`` in ``spec_params`` order (the portfolio kernel convention);
* the ``taic-launch`` block uses expressions over those symbols, so one build serves every shape;
* attributes (EPS, LR, BASE, ...) are compile-time constants rendered from the task's
  ``opspec.json`` defaults (or the caller's values);
* arithmetic in fp32 (rope's angles in fp64), one rounding at the output, NaN/Inf propagating
  the way the tasks' fp64 references do;
* the more involved tasks keep simple parallel forms: attention one warp per query row with an
  online softmax, mamba2 one thread per output (masked terms still multiply x), the KDA
  recurrences one warp per (sequence, head, state row) in fp32.

Implementation ids are ``cuda-sm100.fallback.<task>``, version 1.
"""

from __future__ import annotations

from typing import Mapping

VERSION = 1
CTYPE = {"fp16": "__half", "bf16": "__nv_bfloat16"}

_PRELUDE = """#include <cuda_fp16.h>
#include <cuda_bf16.h>
typedef {ctype} T;
__device__ __forceinline__ float ldf(const T* p, long long i) {{ return (float)p[i]; }}
__device__ __forceinline__ T tof(float v) {{ return T(v); }}
__device__ __forceinline__ float sigm(float v) {{ return 1.0f / (1.0f + expf(-v)); }}
__device__ __forceinline__ float block_sum(float v, float* sh) {{
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += sh[w];
    __syncthreads();
    return t;
}}
__device__ __forceinline__ float block_max(float v, float* sh) {{
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t = fmaxf(t, sh[w]);
    __syncthreads();
    return t;
}}
"""

# Grid-stride element loop over N elements, at most 16 CTAs of 256 threads per SM of a B200.
_ELEM_LAUNCH = "kernel {name} grid=min(ceil_div(N,256),2368) threads=256"


def _unary(expr: str) -> tuple[str, str]:
    body = """extern "C" __global__ void {name}(const T* __restrict__ x, T* __restrict__ y, long long N) {{
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N; i += (long long)gridDim.x * blockDim.x) {{
        const float v = ldf(x, i);
        y[i] = tof(""" + expr + """);
    }}
}}
"""
    return body, _ELEM_LAUNCH


_BODIES: dict[str, tuple[str, str]] = {
    "relu": _unary("v > 0.f ? v : (v != v ? v : 0.f)"),
    "sigmoid": _unary("sigm(v)"),
    "sigmoid_shift": _unary("sigm(v) + 1.0f"),
    "silu": _unary("v * sigm(v)"),
    "swiglu": ("""extern "C" __global__ void {name}(const T* __restrict__ gate, const T* __restrict__ up, T* __restrict__ y, long long N) {{
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N; i += (long long)gridDim.x * blockDim.x) {{
        const float g = ldf(gate, i);
        y[i] = tof(g * sigm(g) * ldf(up, i));
    }}
}}
""", _ELEM_LAUNCH),
    "lion": ("""extern "C" __global__ void {name}(const T* __restrict__ p, const T* __restrict__ g, const T* __restrict__ m,
                                        T* __restrict__ p_out, T* __restrict__ m_out, long long N) {{
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N; i += (long long)gridDim.x * blockDim.x) {{
        const float pv = ldf(p, i), gv = ldf(g, i), mv = ldf(m, i);
        const float c = (float)ATTR_BETA1 * mv + (float)(1.0 - ATTR_BETA1) * gv;
        const float s = c > 0.f ? 1.f : (c < 0.f ? -1.f : 0.f);  /* torch.sign: NaN -> 0 */
        p_out[i] = tof(pv * (float)(1.0 - ATTR_LR * ATTR_WD) - (float)ATTR_LR * s);
        m_out[i] = tof((float)ATTR_BETA2 * mv + (float)(1.0 - ATTR_BETA2) * gv);
    }}
}}
""", _ELEM_LAUNCH),
    "rmsnorm": ("""extern "C" __global__ void {name}(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y, long long M, long long H) {{
    __shared__ float sh[32];
    const long long r = blockIdx.x;
    const T* xr = x + r * H;
    float ss = 0.f;
    for (long long j = threadIdx.x; j < H; j += blockDim.x) {{ const float v = ldf(xr, j); ss += v * v; }}
    ss = block_sum(ss, sh);
    const float inv = rsqrtf(ss / (float)H + (float)ATTR_EPS);
    for (long long j = threadIdx.x; j < H; j += blockDim.x) y[r * H + j] = tof(ldf(xr, j) * inv * ldf(w, j));
}}
""", "kernel {name} grid=M threads=256"),
    "softmax": ("""extern "C" __global__ void {name}(const T* __restrict__ x, T* __restrict__ y, long long M, long long N) {{
    __shared__ float sh[32];
    const T* xr = x + (long long)blockIdx.x * N;
    T* yr = y + (long long)blockIdx.x * N;
    float mx = -INFINITY;
    for (long long j = threadIdx.x; j < N; j += blockDim.x) mx = fmaxf(mx, ldf(xr, j));
    mx = block_max(mx, sh);
    float s = 0.f;
    for (long long j = threadIdx.x; j < N; j += blockDim.x) s += expf(ldf(xr, j) - mx);
    s = block_sum(s, sh);
    for (long long j = threadIdx.x; j < N; j += blockDim.x) yr[j] = tof(expf(ldf(xr, j) - mx) / s);
}}
""", "kernel {name} grid=M threads=256"),
    "reduction_sum": ("""extern "C" __global__ void {name}(const T* __restrict__ x, T* __restrict__ y, long long M, long long N) {{
    __shared__ float sh[32];
    const T* xr = x + (long long)blockIdx.x * N;
    float s = 0.f;
    for (long long j = threadIdx.x; j < N; j += blockDim.x) s += ldf(xr, j);
    s = block_sum(s, sh);
    if (threadIdx.x == 0) y[blockIdx.x] = tof(s);
}}
""", "kernel {name} grid=M threads=256"),
    "gemv": ("""extern "C" __global__ void {name}(const T* __restrict__ A, const T* __restrict__ x, T* __restrict__ y, long long M, long long K) {{
    const long long r = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);  /* one warp per row */
    if (r >= M) return;
    float acc = 0.f;
    for (long long k = threadIdx.x & 31; k < K; k += 32) acc = fmaf(ldf(A, r * K + k), ldf(x, k), acc);
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) y[r] = tof(acc);
}}
""", "kernel {name} grid=ceil_div(M,8) threads=256"),
    "gemm": ("""extern "C" __global__ void {name}(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C, long long M, long long N, long long K) {{
    const long long n = (long long)blockIdx.x * 16 + threadIdx.x, m = (long long)blockIdx.y * 16 + threadIdx.y;
    if (m >= M || n >= N) return;
    float acc = 0.f;
    for (long long k = 0; k < K; ++k) acc = fmaf(ldf(A, m * K + k), ldf(B, k * N + n), acc);
    C[m * N + n] = tof(acc);
}}
""", "kernel {name} grid=ceil_div(N,16),ceil_div(M,16) threads=16,16"),
    "gemm_silu": ("""extern "C" __global__ void {name}(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C, long long M, long long N, long long K) {{
    const long long n = (long long)blockIdx.x * 16 + threadIdx.x, m = (long long)blockIdx.y * 16 + threadIdx.y;
    if (m >= M || n >= N) return;
    float acc = 0.f;
    for (long long k = 0; k < K; ++k) acc = fmaf(ldf(A, m * K + k), ldf(B, k * N + n), acc);
    C[m * N + n] = tof(acc * sigm(acc));
}}
""", "kernel {name} grid=ceil_div(N,16),ceil_div(M,16) threads=16,16"),
    "rope": ("""extern "C" __global__ void {name}(const T* __restrict__ x, T* __restrict__ y, long long B, long long H, long long S, long long D) {{
    const long long half = D / 2, total = B * H * S * half;
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (long long)gridDim.x * blockDim.x) {{
        const long long i = t % half, row = t / half, s = row % S;
        const double ang = (double)s * pow((double)ATTR_BASE, -(double)i / (double)half);
        const float c = (float)cos(ang), sn = (float)sin(ang);
        const float x1 = ldf(x, row * D + i), x2 = ldf(x, row * D + half + i);
        y[row * D + i] = tof(x1 * c - x2 * sn);
        y[row * D + half + i] = tof(x1 * sn + x2 * c);
    }}
}}
""", "kernel {name} grid=min(ceil_div(B*H*S*trunc_div(D,2),256),2368) threads=256"),
    "bitdelta_gemm": ("""extern "C" __global__ void {name}(const T* __restrict__ x, const unsigned int* __restrict__ bits, T* __restrict__ y,
                                        long long M, long long N, long long K) {{
    const long long n = (long long)blockIdx.x * 16 + threadIdx.x, m = (long long)blockIdx.y * 16 + threadIdx.y;
    if (m >= M || n >= N) return;
    float acc = 0.f;
    for (long long k = 0; k < K; ++k) {{
        const unsigned int word = bits[(k >> 5) * N + n];  /* bit j of word (kb, n) is row kb*32 + j: +1 set, -1 clear */
        const float xv = ldf(x, m * K + k);
        acc += ((word >> (k & 31)) & 1u) ? xv : -xv;
    }}
    y[m * N + n] = tof(acc * (float)ATTR_SCALE);
}}
""", "kernel {name} grid=ceil_div(N,16),ceil_div(M,16) threads=16,16"),
    "flash_attention": ("""extern "C" __global__ void {name}(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, T* __restrict__ o,
                                        long long B, long long H, long long S, long long D) {{
    /* One warp per query row, online softmax; lane holds dims lane, lane + 32, ... (D <= 256). */
    const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= B * H * S) return;
    const long long bh = row / S;
    const T* qr = q + row * D;
    const T* kb = k + bh * S * D;
    const T* vb = v + bh * S * D;
    float qv[8], acc[8];
    for (int t = 0; t < 8; ++t) {{
        const long long d = lane + 32 * t;
        qv[t] = d < D ? ldf(qr, d) : 0.f;
        acc[t] = 0.f;
    }}
    float m = -INFINITY, l = 0.f;
    for (long long j = 0; j < S; ++j) {{
        float part = 0.f;
        for (int t = 0; t < 8; ++t) {{
            const long long d = lane + 32 * t;
            if (d < D) part = fmaf(qv[t], ldf(kb, j * D + d), part);
        }}
        for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
        const float s = part * (float)ATTR_SM_SCALE;
        const float mn = fmaxf(m, s);  /* fmaxf drops a NaN s; p = exp(NaN) then poisons the row */
        const float corr = (m == mn) ? 1.f : expf(m - mn);
        const float p = (s == -INFINITY) ? 0.f : expf(s - mn);  /* a -inf score has weight 0 */
        l = l * corr + p;
        for (int t = 0; t < 8; ++t) {{
            const long long d = lane + 32 * t;
            if (d < D) acc[t] = acc[t] * corr + p * ldf(vb, j * D + d);
        }}
        m = mn;
    }}
    for (int t = 0; t < 8; ++t) {{
        const long long d = lane + 32 * t;
        if (d < D) o[row * D + d] = tof(acc[t] / l);
    }}
}}
""", "kernel {name} grid=ceil_div(B*H*S,8) threads=256"),
    "mamba2_chunk_scan": ("""extern "C" __global__ void {name}(const T* __restrict__ x, const T* __restrict__ dt, const T* __restrict__ cs,
                                        const T* __restrict__ Bm, const T* __restrict__ Cm, const T* __restrict__ Dskip,
                                        const T* __restrict__ states, T* __restrict__ y, long long BATCH, long long SEQLEN,
                                        long long NHEADS, long long HEADDIM, long long DSTATE, long long CHUNK, long long NCHUNKS) {{
    const long long total = BATCH * SEQLEN * NHEADS * HEADDIM;
    for (long long o = (long long)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += (long long)gridDim.x * blockDim.x) {{
        const long long p = o % HEADDIM, h = (o / HEADDIM) % NHEADS, t = (o / (HEADDIM * NHEADS)) % SEQLEN;
        const long long b = o / (HEADDIM * NHEADS * SEQLEN);
        const long long c = t / CHUNK, lpos = t % CHUNK, t0 = c * CHUNK;
        const T* csr = cs + ((b * NHEADS + h) * NCHUNKS + c) * CHUNK;
        const float csl = ldf(csr, lpos);
        float acc = 0.f;
        /* Every row of the chunk multiplies x, the masked ones by an exact 0 (a non-finite x
           element makes its whole chunk non-finite, as in the fp64 reference). */
        for (long long sp = 0; sp < CHUNK; ++sp) {{
            const long long ts = t0 + sp;
            float wgt = 0.f;
            if (sp <= lpos) {{
                float cb = 0.f;
                for (long long n = 0; n < DSTATE; ++n) cb = fmaf(ldf(Cm, (b * SEQLEN + t) * DSTATE + n), ldf(Bm, (b * SEQLEN + ts) * DSTATE + n), cb);
                wgt = cb * expf(csl - ldf(csr, sp)) * ldf(dt, (b * SEQLEN + ts) * NHEADS + h);
            }}
            acc = fmaf(wgt, ldf(x, ((b * SEQLEN + ts) * NHEADS + h) * HEADDIM + p), acc);
        }}
        float sc = 0.f;
        for (long long n = 0; n < DSTATE; ++n)
            sc = fmaf(ldf(Cm, (b * SEQLEN + t) * DSTATE + n), ldf(states, (((b * NCHUNKS + c) * NHEADS + h) * HEADDIM + p) * DSTATE + n), sc);
        acc = fmaf(sc, expf(csl), acc);
        acc = fmaf(ldf(Dskip, h), ldf(x, o), acc);
        y[o] = tof(acc);
    }}
}}
""", "kernel {name} grid=min(ceil_div(BATCH*SEQLEN*NHEADS*HEADDIM,256),2368) threads=256"),
}

# The KDA recurrence shared by the fixed-length and the varlen fallbacks: one warp per
# (sequence, head, state row v), lane holding key columns lane, lane + 32, ... (D <= 128).
_KDA_CHAIN = """__device__ void kda_chain(const T* q, const T* k, const T* v, const T* g, const T* beta, const float* A_log,
                          const float* dt_bias, const float* s0, float* s_out, T* out, float scale, long long begin, long long end,
                          long long H, long long D, long long h, long long row) {{
    const int lane = threadIdx.x & 31;
    float st[4];
    for (int t = 0; t < 4; ++t) {{
        const long long c = lane + 32 * t;
        st[t] = c < D ? s0[row * D + c] : 0.f;
    }}
    const float da = expf(A_log[h]);
    for (long long tok = begin; tok < end; ++tok) {{
        const long long base = (tok * H + h) * D;
        float qv[4], kv[4], nq = 0.f, nk = 0.f;
        for (int t = 0; t < 4; ++t) {{
            const long long c = lane + 32 * t;
            qv[t] = c < D ? ldf(q, base + c) : 0.f;
            kv[t] = c < D ? ldf(k, base + c) : 0.f;
            nq = fmaf(qv[t], qv[t], nq);
            nk = fmaf(kv[t], kv[t], nk);
        }}
        for (int off = 16; off > 0; off >>= 1) {{
            nq += __shfl_xor_sync(0xffffffffu, nq, off);
            nk += __shfl_xor_sync(0xffffffffu, nk, off);
        }}
        const float rq = rsqrtf(nq + 1e-6f) * scale, rk = rsqrtf(nk + 1e-6f);
        float dot = 0.f;
        for (int t = 0; t < 4; ++t) {{
            const long long c = lane + 32 * t;
            if (c < D) {{
                const float ld = (float)ATTR_LOWER_BOUND * sigm(da * (ldf(g, base + c) + dt_bias[h * D + c]));
                st[t] *= expf(ld);
                dot = fmaf(st[t], kv[t] * rk, dot);
            }}
        }}
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        const float r = (ldf(v, base + row) - dot) * sigm(ldf(beta, tok * H + h));
        float o = 0.f;
        for (int t = 0; t < 4; ++t) {{
            const long long c = lane + 32 * t;
            if (c < D) {{
                st[t] = fmaf(r, kv[t] * rk, st[t]);
                o = fmaf(st[t], qv[t] * rq, o);
            }}
        }}
        for (int off = 16; off > 0; off >>= 1) o += __shfl_xor_sync(0xffffffffu, o, off);
        if (lane == 0) out[base + row] = tof(o);
    }}
    for (int t = 0; t < 4; ++t) {{
        const long long c = lane + 32 * t;
        if (c < D) s_out[row * D + c] = st[t];
    }}
}}
"""

_BODIES["varlen_kda"] = (_KDA_CHAIN + """extern "C" __global__ void {name}(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
        const T* __restrict__ g, const T* __restrict__ beta, const float* __restrict__ A_log, const float* __restrict__ dt_bias,
        const float* __restrict__ initial_state, const int* __restrict__ cu_seqlens, const float* __restrict__ scale,
        T* __restrict__ output, float* __restrict__ final_state, float* log_decay_tab, float* token_stats, unsigned int* work_items,
        int* item_counts, int* handoff_flags, float* handoff_states, long long H, long long D) {{
    /* Warps cover num_seqs * H * D rows exactly (D % 8 == 0); a sequence whose offsets hold the
       negative capacity sentinel is left untouched. */
    const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const long long row = w % D, h = (w / D) % H, s = w / (D * H);
    const long long begin = cu_seqlens[s], end = cu_seqlens[s + 1];
    if (begin < 0 || end < 0 || end < begin) return;
    const long long off = (s * H + h) * D * D;
    kda_chain(q, k, v, g, beta, A_log, dt_bias, initial_state + off, final_state + off, output, scale[0], begin, end, H, D, h, row);
}}
""", "kernel {name} grid=ceil_div(num_seqs*H*D,8) threads=256")

_BODIES["kda"] = (_KDA_CHAIN + """extern "C" __global__ void {name}(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
        const T* __restrict__ g, const T* __restrict__ beta, const float* __restrict__ A_log, const float* __restrict__ dt_bias,
        const float* __restrict__ initial_state, const float* __restrict__ scale, T* __restrict__ output,
        float* __restrict__ final_state, unsigned int* __restrict__ work_items, int* __restrict__ item_counts,
        float* handoff_states, long long N, long long H, long long D) {{
    const long long w = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (w == 0 && (threadIdx.x & 31) == 0) {{
        /* The host program's work list: one piece [0, N), two empty ones. */
        work_items[0] = 0u; work_items[1] = (unsigned int)N; work_items[2] = (unsigned int)N;
        work_items[3] = 0u; work_items[4] = (unsigned int)N; work_items[5] = 0u;
        item_counts[0] = 1;
    }}
    if (w >= H * D) return;
    const long long row = w % D, h = w / D;
    const long long off = h * D * D;
    kda_chain(q, k, v, g, beta, A_log, dt_bias, initial_state + off, final_state + off, output, scale[0], 0, N, H, D, h, row);
}}
""", "kernel {name} grid=ceil_div(H*D,8) threads=256")

# Attribute defaults of tasks/<task>/opspec.json (used when the caller passes none).
ATTR_DEFAULTS: dict[str, dict[str, float]] = {
    "rmsnorm": {"EPS": 1e-6},
    "lion": {"LR": 0.001, "WD": 0.1, "BETA1": 0.9, "BETA2": 0.99},
    "rope": {"BASE": 10000.0},
    "bitdelta_gemm": {"SCALE": 0.02},
    "flash_attention": {"SM_SCALE": 0.125},
    "kda": {"LOWER_BOUND": -5.0},
    "varlen_kda": {"LOWER_BOUND": -5.0},
}

TASKS = tuple(sorted(_BODIES))


def implementation_id(task: str) -> str:
    return f"cuda-sm100.fallback.{task}"


def kernel_name(task: str) -> str:
    return f"fallback_{task}"


def render(task: str, dtype: str, attrs: Mapping[str, float] | None = None) -> str:
    """The fallback source of ``task`` for storage dtype ``dtype`` (``fp16``/``bf16``)."""
    if task not in _BODIES:
        raise KeyError(f"no registered CUDA fallback for task {task!r}; registered: {list(TASKS)}")
    if dtype not in CTYPE:
        raise ValueError(f"fallbacks take fp16/bf16 storage, got {dtype!r}")
    values = dict(ATTR_DEFAULTS.get(task, {}))
    values.update(attrs or {})
    body, launch = _BODIES[task]
    name = kernel_name(task)
    defines = "".join(f"#define ATTR_{k} ({float(v)!r})\n" for k, v in sorted(values.items()))
    return (
        f"// {implementation_id(task)} v{VERSION}: naive fallback of tasks/{task} ({dtype}).\n"
        + _PRELUDE.format(ctype=CTYPE[dtype]) + defines + body.format(name=name)
        + "/* taic-launch\n" + launch.format(name=name) + "\n*/\n"
    )
