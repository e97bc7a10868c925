// Shared helpers of the sm_100a kernels: status reporting, dtype traits, vector IO.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/sfcuda.h"

namespace sf {

// Write a formatted message into the caller's error buffer (may be NULL/0) and return `code`.
static inline int fail(int code, char* err, uint64_t cap, const char* fmt, ...) {
    if (err && cap) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(err, (size_t)cap, fmt, ap);
        va_end(ap);
    }
    return code;
}

// Map the last CUDA runtime error (after an asynchronous launch) to SF_EDEVICE.
static inline int check_launch(const char* what, char* err, uint64_t cap) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        return fail(SF_EDEVICE, err, cap, "%s: %s", what, cudaGetErrorString(e));
    }
    return SF_OK;
}

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Number of SMs of the current device (cached per device).
int sm_count();

// CTAs of `kernel` resident on one SM at `threads` threads and `smem` bytes of dynamic shared
// memory (the occupancy calculator; at least 1).  Grid-stride kernels size their grid as
// sm_count() x this, so the whole grid is one wave and every CTA gets the same share.
template <typename K>
int resident_ctas(K kernel, int threads, size_t smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess || n < 1) {
        cudaGetLastError();
        n = 1;
    }
    return n;
}

template <typename T> struct Dt;
template <> struct Dt<__half> {
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Dt<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// 8 x 16-bit values packed in one 128-bit word.
template <typename T>
struct alignas(16) Vec8 {
    T v[8];
};

template <typename T>
__device__ __forceinline__ Vec8<T> ld_global_nc_v8(const T* p) {
    uint4 raw;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(raw.x), "=r"(raw.y), "=r"(raw.z), "=r"(raw.w)
                 : "l"(p));
    Vec8<T> out;
    *reinterpret_cast<uint4*>(&out) = raw;
    return out;
}

template <typename T>
__device__ __forceinline__ void st_global_v8(T* p, const Vec8<T>& v) {
    const uint4 raw = *reinterpret_cast<const uint4*>(&v);
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(raw.x), "r"(raw.y),
                 "r"(raw.z), "r"(raw.w)
                 : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Packed fp32 pair arithmetic (sm_100: one FFMA2 / FMUL2 / FADD2 instruction for two values).
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
    float2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(reinterpret_cast<uint64_t&>(d))
        : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)), "l"(reinterpret_cast<const uint64_t&>(c)));
    return d;
}
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
    float2 d;
    asm("mul.rn.f32x2 %0, %1, %2;"
        : "=l"(reinterpret_cast<uint64_t&>(d))
        : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)));
    return d;
}
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
    float2 d;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(reinterpret_cast<uint64_t&>(d))
        : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)));
    return d;
}
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

// 2^x with the hardware approximation, subnormal results flushed to zero (a single MUFU op; the
// non-flushing form adds range handling around it).
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// e^-|x| for the sigmoid below: 2^(-|x| log2 e), flushed to 0 below 2^-126 (|x| > 87.3).
__device__ __forceinline__ float exp_neg_abs(float x) { return ex2_ftz(fabsf(x) * -1.4426950408889634f); }

// sigmoid(x) = 1 / (1 + e^-x) with one MUFU operation per element and no branch.
// With t = e^-|x| in (0, 1] the denominator d = 1 + t lies in [1, 2], so 1/d comes from the
// Newton-Raphson division seed 24/17 - 8/17 d (maximum relative error 1/17 on [1, 2]) and three
// Newton steps r += r (1 - d r) (error 1/17 -> 2^-8.2 -> 2^-16.4 -> below fp32 rounding); then
// sigmoid(x) = 1/d for x >= 0 and t/d = e^x / (1 + e^x) for x < 0.  Within 3 fp32 ulps of the
// exact value for |x| <= 80; for x < -87.3 t flushes to 0 and so does the result (the exact value
// is below 2^-126 there, under every tolerance of a 16-bit output).  NaN propagates through t;
// +Inf gives 1 and -Inf gives +0.  sigmoid2_nr does the same for a pair with packed arithmetic
// (written with nd = -d so that every step is one FFMA2).
__device__ __forceinline__ float sigmoid_nr(float x) {
    const float t = exp_neg_abs(x);
    const float d = 1.0f + t;
    float r = fmaf(-8.0f / 17.0f, d, 24.0f / 17.0f);
#pragma unroll
    for (int i = 0; i < 3; ++i) r = fmaf(r, fmaf(-d, r, 1.0f), r);
    return x >= 0.f ? r : t * r;
}

__device__ __forceinline__ float2 sigmoid2_nr(float2 x) {
    const float2 t = make_float2(exp_neg_abs(x.x), exp_neg_abs(x.y));
    const float2 nd = f2_fma(t, f2(-1.0f), f2(-1.0f));  // -(1 + t)
    float2 r = f2_fma(f2(8.0f / 17.0f), nd, f2(24.0f / 17.0f));
#pragma unroll
    for (int i = 0; i < 3; ++i) r = f2_fma(r, f2_fma(nd, r, f2(1.0f)), r);
    const float2 tr = f2_mul(t, r);
    return make_float2(x.x >= 0.f ? r.x : tr.x, x.y >= 0.f ? r.y : tr.y);
}

// Two 16-bit values packed in a 32-bit word <-> a float pair.
template <typename T> struct Pair;
template <> struct Pair<__half> {
    static __device__ __forceinline__ float2 to_f2(uint32_t w) { return __half22float2(*reinterpret_cast<const __half2*>(&w)); }
    static __device__ __forceinline__ uint32_t from_f2(float2 v) {
        const __half2 h = __floats2half2_rn(v.x, v.y);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
};
template <> struct Pair<__nv_bfloat16> {
    static __device__ __forceinline__ float2 to_f2(uint32_t w) {
        return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    }
    static __device__ __forceinline__ uint32_t from_f2(float2 v) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
};

}  // namespace sf

// Per-op launchers (defined in the op's .cu file) used by sf_run_op.
int sf_rmsnorm_launch(const void* x, const void* w, void* y, int64_t rows, int64_t hidden, float eps,
                      int32_t dtype, int32_t variant, cudaStream_t stream, char* err, uint64_t cap);
int sf_gemm_nt_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, int32_t variant,
                      cudaStream_t s, char* err, uint64_t cap);
int sf_gemm_nn_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, int32_t variant,
                      void* workspace, uint64_t workspace_bytes, cudaStream_t s, char* err, uint64_t cap);
int sf_silu_launch(const void* x, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err, uint64_t cap);
int sf_swiglu_launch(const void* gate, const void* up, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s,
                     char* err, uint64_t cap);
int sf_relu_launch(const void* x, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err, uint64_t cap);
int sf_sigmoid_launch(const void* x, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err, uint64_t cap);
int sf_sigmoid_shift_launch(const void* x, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err,
                            uint64_t cap);
int sf_lion_launch(const void* p, const void* g, const void* m, void* p_out, void* m_out, int64_t n, double lr, double wd,
                   double beta1, double beta2, int32_t dtype, int32_t variant, cudaStream_t s, char* err, uint64_t cap);
int sf_gemv_launch(const void* A, const void* x, void* y, int64_t M, int64_t K, int32_t dtype, int32_t variant, cudaStream_t s,
                   char* err, uint64_t cap);
int sf_gemm_silu_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, int32_t variant,
                        void* workspace, uint64_t workspace_bytes, cudaStream_t s, char* err, uint64_t cap);
int sf_softmax_launch(const void* x, void* y, int64_t m, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err,
                      uint64_t cap);
int sf_reduction_sum_launch(const void* x, void* y, int64_t m, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s,
                            char* err, uint64_t cap);
int sf_rope_launch(const void* x, void* y, int64_t B, int64_t H, int64_t S, int64_t D, double base, int32_t dtype, int32_t variant,
                   cudaStream_t st, char* err, uint64_t cap);
int sf_bitdelta_launch(const void* x, const void* bits, void* y, int64_t M, int64_t N, int64_t K, float scale, int32_t dtype,
                       int32_t variant, cudaStream_t st, char* err, uint64_t cap);
int sf_bitdelta_base_launch(const void* x, const void* w_base, const void* s_words, const void* alpha, void* y, int64_t M, int64_t N,
                            int64_t K, int32_t dtype, int32_t variant, cudaStream_t st, char* err, uint64_t cap);
int sf_bitdelta_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream);
int sf_attention_launch(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H, int64_t S, int64_t D, float scale,
                        int32_t causal, int32_t dtype, int32_t variant, cudaStream_t st, char* err, uint64_t cap);
int sf_attention_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream);
int sf_kda_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log, const void* dt_bias,
                  const void* initial_state, const void* cu_seqlens, const void* scale, void* out, void* final_state, int64_t N,
                  int64_t H, int64_t D, float lower_bound, int32_t dtype, int32_t variant, int64_t total_tokens, void* workspace,
                  uint64_t workspace_bytes, cudaStream_t st, char* err, uint64_t cap);
int sf_kda_fixed_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
                        const void* dt_bias, const void* initial_state, const void* scale, void* out, void* final_state,
                        void* work_items, void* item_counts, int64_t N, int64_t H, int64_t D, float lower_bound, int32_t dtype,
                        int32_t variant, cudaStream_t st, char* err, uint64_t cap);
int sf_kda_task_chunk_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
                             const void* dt_bias, const void* initial_state, const void* cu_seqlens, const void* scale, void* out,
                             void* final_state, int64_t N, int64_t H, int64_t D, float lower_bound, int32_t dtype, cudaStream_t st,
                             char* err, uint64_t cap);
int sf_kda_gated_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                        const void* initial_state, void* out, void* final_state, int64_t N, int64_t H, int64_t D, float scale,
                        int32_t dtype, int32_t variant, int64_t total_tokens, void* workspace, uint64_t workspace_bytes,
                        cudaStream_t st, char* err, uint64_t cap);
int sf_kda_gated_chunk_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                              const void* initial_state, void* out, void* final_state, int64_t N, int64_t H, int64_t D, float scale,
                              int32_t dtype, cudaStream_t st, char* err, uint64_t cap);
int sf_kda_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream);
int sf_kda_gated_c32_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                            const void* initial_state, void* out, void* final_state, int64_t N, int64_t H, int64_t D, float scale,
                            int32_t dtype, cudaStream_t st, char* err, uint64_t cap);
int sf_kda32_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream);
uint64_t sf_kda_gated_split_workspace(int64_t total_tokens, int64_t nseq, int64_t H, int64_t D);
int sf_kda_gated_split_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                              const void* initial_state, void* out, void* final_state, int64_t N, int64_t total_tokens, int64_t H,
                              int64_t D, float scale, int32_t dtype, void* workspace, uint64_t workspace_bytes, cudaStream_t st,
                              char* err, uint64_t cap);
int sf_kda_task_split_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
                             const void* dt_bias, const void* initial_state, const void* cu_seqlens, const void* scale, void* out,
                             void* final_state, int64_t N, int64_t total_tokens, int64_t H, int64_t D, float lower_bound,
                             int32_t dtype, void* workspace, uint64_t workspace_bytes, cudaStream_t st, char* err, uint64_t cap);
int sf_kda_split_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream);
int sf_mamba2_launch(const void* x, const void* dt, const void* cs, const void* bm, const void* cm, const void* dskip, const void* states,
                     void* y, int64_t B, int64_t L, int64_t H, int64_t P, int64_t N, int64_t C, int32_t dtype, int32_t variant,
                     cudaStream_t st, char* err, uint64_t cap);
int sf_mamba2_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream);
