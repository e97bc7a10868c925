// Row-wise task operators for sm_100a: softmax and reduction_sum over the last axis of [M, N].
//
//   softmax        y[r,:] = exp(x[r,:] - max) / sum(exp(x[r,:] - max))   tasks/softmax/reference.py:104-106
//   reduction_sum  y[r]   = sum(x[r,:])                                  tasks/reduction_sum/reference.py:104-106
//
// HBM-bound.  One CTA per row; on the fast path (N % 8 == 0, aligned bases, N <= 65536) each
// thread keeps its 16-byte vectors of the row in registers, so x is read from HBM once.  The
// row max propagates NaN (a NaN anywhere makes the row NaN, like the fp64 reference), an +Inf
// makes exp(inf - inf) = NaN and so a NaN row, -Inf entries get weight 0.  Sums accumulate in
// fp32 (per-thread partials, then a warp/CTA tree).  General rows take a strided multi-pass loop.
#include "sf_common.cuh"

namespace {

constexpr int kMaxWarps = 32;

__device__ __forceinline__ float nan_max(float a, float b) { return (b > a || b != b) ? b : a; }

__device__ __forceinline__ float warp_nan_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = nan_max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Reduce `v` over the CTA with op (0 = sum, 1 = NaN-propagating max); `red` holds kMaxWarps+1.
template <int OP>
__device__ __forceinline__ float block_reduce(float v, float* red) {
    v = OP == 0 ? sf::warp_sum(v) : warp_nan_max(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = (blockDim.x + 31) >> 5;
    __syncthreads();  // red may still be read by a previous reduction
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nwarps ? red[lane] : (OP == 0 ? 0.f : -INFINITY);
        t = OP == 0 ? sf::warp_sum(t) : warp_nan_max(t);
        if (lane == 0) red[kMaxWarps] = t;
    }
    __syncthreads();
    return red[kMaxWarps];
}

template <typename T, int NV>
__global__ void __launch_bounds__(1024) softmax_vec_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
    __shared__ float red[kMaxWarps + 1];
    const int64_t row = blockIdx.x;
    const int64_t nvec = n >> 3;
    const T* xr = x + row * n;
    T* yr = y + row * n;
    float f[NV][8];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t idx = (int64_t)threadIdx.x + (int64_t)i * blockDim.x;
        if (idx < nvec) {
            const sf::Vec8<T> v = sf::ld_global_nc_v8<T>(xr + idx * 8);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                f[i][j] = sf::Dt<T>::to_f(v.v[j]);
                m = nan_max(m, f[i][j]);
            }
        }
    }
    m = block_reduce<1>(m, red);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t idx = (int64_t)threadIdx.x + (int64_t)i * blockDim.x;
        if (idx < nvec) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                f[i][j] = __expf(f[i][j] - m);
                s += f[i][j];
            }
        }
    }
    s = block_reduce<0>(s, red);
    const float inv = 1.0f / s;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t idx = (int64_t)threadIdx.x + (int64_t)i * blockDim.x;
        if (idx < nvec) {
            sf::Vec8<T> o;
#pragma unroll
            for (int j = 0; j < 8; ++j) o.v[j] = sf::Dt<T>::from_f(f[i][j] * inv);
            sf::st_global_v8<T>(yr + idx * 8, o);
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(256) softmax_generic_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
    __shared__ float red[kMaxWarps + 1];
    const int64_t row = blockIdx.x;
    const T* xr = x + row * n;
    T* yr = y + row * n;
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) m = nan_max(m, sf::Dt<T>::to_f(xr[i]));
    m = block_reduce<1>(m, red);
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += __expf(sf::Dt<T>::to_f(xr[i]) - m);
    s = block_reduce<0>(s, red);
    const float inv = 1.0f / s;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) yr[i] = sf::Dt<T>::from_f(__expf(sf::Dt<T>::to_f(xr[i]) - m) * inv);
}

template <typename T, int NV>
__global__ void __launch_bounds__(1024) rowsum_vec_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
    __shared__ float red[kMaxWarps + 1];
    const int64_t row = blockIdx.x;
    const int64_t nvec = n >> 3;
    const T* xr = x + row * n;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t idx = (int64_t)threadIdx.x + (int64_t)i * blockDim.x;
        if (idx < nvec) {
            const sf::Vec8<T> v = sf::ld_global_nc_v8<T>(xr + idx * 8);
            float p = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) p += sf::Dt<T>::to_f(v.v[j]);
            s += p;
        }
    }
    s = block_reduce<0>(s, red);
    if (threadIdx.x == 0) y[row] = sf::Dt<T>::from_f(s);
}

template <typename T>
__global__ void __launch_bounds__(256) rowsum_generic_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
    __shared__ float red[kMaxWarps + 1];
    const int64_t row = blockIdx.x;
    const T* xr = x + row * n;
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += sf::Dt<T>::to_f(xr[i]);
    s = block_reduce<0>(s, red);
    if (threadIdx.x == 0) y[row] = sf::Dt<T>::from_f(s);
}

// Vectors per thread: the smallest of 1/2/4/8 giving <= 128 threads (8 may use up to 1024), so up
// to 16 rows are resident per SM and more of each row's bytes are in flight per thread.
int pick_nv(int64_t n) {
    const int64_t nvec = n / 8;
    for (int cand : {1, 2, 4, 8}) {
        const int64_t threads = (nvec + cand - 1) / cand;
        if (threads <= 128 || (cand == 8 && threads <= 1024)) return cand;
    }
    return 0;
}

template <typename T, bool SOFTMAX>
int launch_t(const void* x, void* y, int64_t m, int64_t n, int32_t variant, cudaStream_t s, char* err, uint64_t cap) {
    const bool vec_ok = variant != 2 && n % 8 == 0 && sf::aligned16(x) && (!SOFTMAX || sf::aligned16(y));
    const int nv = vec_ok ? pick_nv(n) : 0;
    if (m > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "row op: M too large");
    const dim3 grid((unsigned)m);
    if (nv > 0) {
        int64_t threads = (n / 8 + nv - 1) / nv;
        threads = ((threads + 31) / 32) * 32;
        const dim3 block((unsigned)threads);
#define SF_ROW_CASE(NVV)                                                                                     \
    case NVV:                                                                                                \
        if (SOFTMAX) softmax_vec_kernel<T, NVV><<<grid, block, 0, s>>>((const T*)x, (T*)y, n);              \
        else rowsum_vec_kernel<T, NVV><<<grid, block, 0, s>>>((const T*)x, (T*)y, n);                       \
        break;
        switch (nv) {
            SF_ROW_CASE(1)
            SF_ROW_CASE(2)
            SF_ROW_CASE(4)
            SF_ROW_CASE(8)
        }
#undef SF_ROW_CASE
    } else {
        if (SOFTMAX) softmax_generic_kernel<T><<<grid, 256, 0, s>>>((const T*)x, (T*)y, n);
        else rowsum_generic_kernel<T><<<grid, 256, 0, s>>>((const T*)x, (T*)y, n);
    }
    return sf::check_launch(SOFTMAX ? "softmax launch" : "reduction_sum launch", err, cap);
}

template <bool SOFTMAX>
int launch(const void* x, void* y, int64_t m, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err, uint64_t cap) {
    const char* name = SOFTMAX ? "softmax" : "reduction_sum";
    if (m < 0 || n < 1) return sf::fail(SF_EINVAL, err, cap, "%s: need M >= 0 and N >= 1", name);
    if (m == 0) return SF_OK;
    if (!x || !y) return sf::fail(SF_EINVAL, err, cap, "%s: null tensor pointer", name);
    if (dtype == SF_DTYPE_F16) return launch_t<__half, SOFTMAX>(x, y, m, n, variant, s, err, cap);
    if (dtype == SF_DTYPE_BF16) return launch_t<__nv_bfloat16, SOFTMAX>(x, y, m, n, variant, s, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "%s: dtype %d is not fp16/bf16", name, dtype);
}

}  // namespace

int sf_softmax_launch(const void* x, void* y, int64_t m, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err,
                      uint64_t cap) {
    return launch<true>(x, y, m, n, dtype, variant, s, err, cap);
}

int sf_reduction_sum_launch(const void* x, void* y, int64_t m, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s,
                            char* err, uint64_t cap) {
    return launch<false>(x, y, m, n, dtype, variant, s, err, cap);
}

extern "C" int sf_softmax(const void* x, void* y, int64_t m, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_softmax_launch(x, y, m, n, dtype, 0, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_reduction_sum(const void* x, void* y, int64_t m, int64_t n, int32_t dtype, void* stream, char* err,
                                uint64_t cap) {
    return sf_reduction_sum_launch(x, y, m, n, dtype, 0, (cudaStream_t)stream, err, cap);
}
