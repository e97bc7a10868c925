// Element-wise task operators for sm_100a: silu and swiglu.
//
//   silu   y = x * sigmoid(x)              tasks/silu/reference.py:105-108
//   swiglu y = gate * sigmoid(gate) * up   tasks/swiglu/reference.py:109-113
//
// HBM-bound (2 or 3 streams of 16-bit elements, a handful of flops each).  A grid-stride loop of
// 16-byte vector loads/stores over a grid of 8 CTAs per SM; the element tail and unaligned bases
// take a scalar loop.  sigmoid is evaluated in fp32 as 1 / (1 + exp(-x)), which maps +-Inf and NaN
// the way the fp64 reference does (sigmoid(-inf) = 0, so silu(-inf) = -inf * 0 = NaN).
#include "sf_common.cuh"

namespace {

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }

template <typename T, bool GLU>
__global__ void __launch_bounds__(256) act_kernel(const T* __restrict__ x, const T* __restrict__ up, T* __restrict__ y,
                                                  int64_t n, bool vec) {
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t done = 0;
    if (vec) {
        const int64_t nv = n >> 3;
        auto apply = [&](const sf::Vec8<T>& a, const sf::Vec8<T>& u, int64_t i) {
            sf::Vec8<T> o;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float f = sf::Dt<T>::to_f(a.v[j]);
                float r = f * sigmoidf_(f);
                if (GLU) r *= sf::Dt<T>::to_f(u.v[j]);
                o.v[j] = sf::Dt<T>::from_f(r);
            }
            sf::st_global_v8<T>(y + i * 8, o);
        };
        // silu: two independent vectors per thread and step, so twice the bytes are in flight
        // (swiglu already has two input streams per vector).
        int64_t i = tid;
        for (; !GLU && i + stride < nv; i += 2 * stride) {
            const sf::Vec8<T> a0 = sf::ld_global_nc_v8<T>(x + i * 8);
            const sf::Vec8<T> a1 = sf::ld_global_nc_v8<T>(x + (i + stride) * 8);
            sf::Vec8<T> u0, u1;
            if (GLU) {
                u0 = sf::ld_global_nc_v8<T>(up + i * 8);
                u1 = sf::ld_global_nc_v8<T>(up + (i + stride) * 8);
            }
            apply(a0, u0, i);
            apply(a1, u1, i + stride);
        }
        for (; i < nv; i += stride) {
            sf::Vec8<T> u0;
            if (GLU) u0 = sf::ld_global_nc_v8<T>(up + i * 8);
            apply(sf::ld_global_nc_v8<T>(x + i * 8), u0, i);
        }
        done = nv * 8;
    }
    for (int64_t i = done + tid; i < n; i += stride) {
        const float f = sf::Dt<T>::to_f(x[i]);
        float r = f * sigmoidf_(f);
        if (GLU) r *= sf::Dt<T>::to_f(up[i]);
        y[i] = sf::Dt<T>::from_f(r);
    }
}

template <typename T, bool GLU>
int launch_t(const void* x, const void* up, void* y, int64_t n, int32_t variant, cudaStream_t s, char* err, uint64_t cap) {
    const bool vec = variant != 2 && sf::aligned16(x) && sf::aligned16(y) && (!GLU || sf::aligned16(up));
    const int64_t work = vec ? (n + 7) / 8 : n;
    int64_t blocks = (work + 255) / 256;
    const int64_t cap_blocks = (int64_t)sf::sm_count() * 8;
    if (blocks > cap_blocks) blocks = cap_blocks;
    if (blocks < 1) blocks = 1;
    act_kernel<T, GLU><<<(unsigned)blocks, 256, 0, s>>>((const T*)x, (const T*)up, (T*)y, n, vec);
    return sf::check_launch(GLU ? "swiglu launch" : "silu launch", err, cap);
}

template <bool GLU>
int launch(const void* x, const void* up, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err,
           uint64_t cap) {
    const char* name = GLU ? "swiglu" : "silu";
    if (n < 0) return sf::fail(SF_EINVAL, err, cap, "%s: negative size", name);
    if (n == 0) return SF_OK;
    if (!x || !y || (GLU && !up)) return sf::fail(SF_EINVAL, err, cap, "%s: null tensor pointer", name);
    if (dtype == SF_DTYPE_F16) return launch_t<__half, GLU>(x, up, y, n, variant, s, err, cap);
    if (dtype == SF_DTYPE_BF16) return launch_t<__nv_bfloat16, GLU>(x, up, y, n, variant, s, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "%s: dtype %d is not fp16/bf16", name, dtype);
}

}  // namespace

int sf_silu_launch(const void* x, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err, uint64_t cap) {
    return launch<false>(x, nullptr, y, n, dtype, variant, s, err, cap);
}

int sf_swiglu_launch(const void* gate, const void* up, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s,
                     char* err, uint64_t cap) {
    return launch<true>(gate, up, y, n, dtype, variant, s, err, cap);
}

extern "C" int sf_silu(const void* x, void* y, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_silu_launch(x, y, n, dtype, 0, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_swiglu(const void* gate, const void* up, void* y, int64_t n, int32_t dtype, void* stream, char* err,
                         uint64_t cap) {
    return sf_swiglu_launch(gate, up, y, n, dtype, 0, (cudaStream_t)stream, err, cap);
}
