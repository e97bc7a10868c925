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
  the way the tasks' fp64 references do.

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
}

# Attribute defaults of tasks/<task>/opspec.json (used when the caller passes none).
ATTR_DEFAULTS: dict[str, dict[str, float]] = {
    "rmsnorm": {"EPS": 1e-6},
    "lion": {"LR": 0.001, "WD": 0.1, "BETA1": 0.9, "BETA2": 0.99},
    "rope": {"BASE": 10000.0},
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
