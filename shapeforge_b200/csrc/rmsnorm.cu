// rmsnorm for sm_100a: y[r,:] = x[r,:] * rsqrt(mean(x[r,:]^2) + eps) * w.
//
// Semantics follow tasks/rmsnorm/reference.py:110-115 (fp64 oracle, one rounding at the output)
// and opspec.json:5 (fp32 accumulation).  The op is HBM-bound: 2*R*H bytes of x and y plus
// 2*H of w per call, ~1 flop/byte.  Design:
//   * rows of at most 1024 elements (hidden % 8 == 0, aligned): one warp per row, shuffle-only
//     reduction (rmsnorm_warp_kernel): a CTA and two barriers per 2 KB row made 4096 x 1024 run at
//     half of HBM bandwidth;
//   * fast path (hidden % 8 == 0, 16-byte aligned bases): one CTA per row, each thread keeps
//     NV 128-bit vectors of the row in registers, so x is read from HBM exactly once; the
//     sum of squares is a warp-shuffle + shared-memory reduction in fp32; w is read through
//     the read-only path (it stays L2/L1 resident across rows);
//   * general path (any hidden, any alignment): one CTA per row, two strided passes (the
//     second pass re-reads the row from L1/L2).
#include "sf_common.cuh"

#include <algorithm>

namespace {

constexpr int kMaxWarps = 32;

template <typename T>
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = sf::warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = (blockDim.x + 31) >> 5;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nwarps ? red[lane] : 0.f;
        t = sf::warp_sum(t);
        if (lane == 0) red[kMaxWarps] = t;
    }
    __syncthreads();
    return red[kMaxWarps];
}

// NV vectors of 8 elements per thread; threads past the row's vector count are masked.
template <typename T, int NV>
__global__ void __launch_bounds__(1024) rmsnorm_vec_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                           T* __restrict__ y, int64_t hidden, float eps) {
    __shared__ float red[kMaxWarps + 1];
    const int64_t row = blockIdx.x;
    const int64_t nvec = hidden >> 3;
    const T* xr = x + row * hidden;
    T* yr = y + row * hidden;
    sf::Vec8<T> v[NV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t idx = (int64_t)threadIdx.x + (int64_t)i * blockDim.x;
        if (idx < nvec) {
            v[i] = sf::ld_global_nc_v8<T>(xr + idx * 8);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float f = sf::Dt<T>::to_f(v[i].v[j]);
                ss = fmaf(f, f, ss);
            }
        }
    }
    const float total = block_sum<T>(ss, red);
    const float r = rsqrtf(total / (float)hidden + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t idx = (int64_t)threadIdx.x + (int64_t)i * blockDim.x;
        if (idx < nvec) {
            const sf::Vec8<T> wv = *reinterpret_cast<const sf::Vec8<T>*>(w + idx * 8);
            sf::Vec8<T> o;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                o.v[j] = sf::Dt<T>::from_f(sf::Dt<T>::to_f(v[i].v[j]) * r * sf::Dt<T>::to_f(wv.v[j]));
            }
            sf::st_global_v8<T>(yr + idx * 8, o);
        }
    }
}

// Rows of at most 1024 elements: one warp per row, NVW 16-byte vectors per lane held packed in
// registers, the sum of squares reduced with shuffles only (no shared memory, no CTA barrier); a
// row's x loads are issued before its w loads (w stays in L1/L2).  Rows are visited
// grid-stride by the warps of a single wave of 8-warp CTAs.
template <typename T, int NVW>
__global__ void __launch_bounds__(256) rmsnorm_warp_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                                                           int64_t rows, int64_t hidden, float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t nvec = hidden >> 3;
    const int64_t wstride = (int64_t)gridDim.x * 8;
    for (int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); row < rows; row += wstride) {
        const T* xr = x + row * hidden;
        sf::Vec8<T> v[NVW], wv[NVW];
        // x first (HBM), then w (L1/L2-resident): w's latency overlaps x's instead of preceding it.
#pragma unroll
        for (int i = 0; i < NVW; ++i) {
            const int64_t idx = lane + 32 * i;
            if (idx < nvec) v[i] = sf::ld_global_nc_v8<T>(xr + idx * 8);
        }
#pragma unroll
        for (int i = 0; i < NVW; ++i) {
            const int64_t idx = lane + 32 * i;
            if (idx < nvec) wv[i] = *reinterpret_cast<const sf::Vec8<T>*>(w + idx * 8);
        }
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < NVW; ++i) {
            const int64_t idx = lane + 32 * i;
            if (idx < nvec) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float f = sf::Dt<T>::to_f(v[i].v[j]);
                    ss = fmaf(f, f, ss);
                }
            }
        }
        const float r = rsqrtf(sf::warp_sum(ss) / (float)hidden + eps);
        T* yr = y + row * hidden;
#pragma unroll
        for (int i = 0; i < NVW; ++i) {
            const int64_t idx = lane + 32 * i;
            if (idx < nvec) {
                sf::Vec8<T> o;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    o.v[j] = sf::Dt<T>::from_f(sf::Dt<T>::to_f(v[i].v[j]) * r * sf::Dt<T>::to_f(wv[i].v[j]));
                sf::st_global_v8<T>(yr + idx * 8, o);
            }
        }
    }
}

template <typename T, int NVW>
int launch_warp_rows(const T* x, const T* w, T* y, int64_t rows, int64_t hidden, float eps, cudaStream_t stream, char* err,
                     uint64_t cap) {
    static const int resident = sf::resident_ctas(rmsnorm_warp_kernel<T, NVW>, 256, 0);
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, (int64_t)sf::sm_count() * resident));
    rmsnorm_warp_kernel<T, NVW><<<(unsigned)blocks, 256, 0, stream>>>(x, w, y, rows, hidden, eps);
    return sf::check_launch("rmsnorm launch", err, cap);
}

template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_generic_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                              T* __restrict__ y, int64_t hidden, float eps) {
    __shared__ float red[kMaxWarps + 1];
    const int64_t row = blockIdx.x;
    const T* xr = x + row * hidden;
    T* yr = y + row * hidden;
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
        const float f = sf::Dt<T>::to_f(xr[i]);
        ss = fmaf(f, f, ss);
    }
    const float total = block_sum<T>(ss, red);
    const float r = rsqrtf(total / (float)hidden + eps);
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
        yr[i] = sf::Dt<T>::from_f(sf::Dt<T>::to_f(xr[i]) * r * sf::Dt<T>::to_f(w[i]));
    }
}

template <typename T>
int launch_typed(const T* x, const T* w, T* y, int64_t rows, int64_t hidden, float eps, int32_t variant,
                 cudaStream_t stream, char* err, uint64_t cap) {
    if (rows > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "rmsnorm: rows %lld exceeds the grid limit", (long long)rows);
    const bool vec_ok = (hidden % 8 == 0) && sf::aligned16(x) && sf::aligned16(w) && sf::aligned16(y);
    const int64_t nvec = hidden / 8;
    // Rows of <= 1024 elements: a warp per row (variant 0; variant 1 keeps the CTA-per-row kernel).
    // Longer rows stay on one CTA per row: eight vectors per lane take 124-158 registers, one CTA
    // per SM, too few bytes in flight.
    if (vec_ok && variant == 0 && nvec <= 128) {
        if (nvec <= 32) return launch_warp_rows<T, 1>(x, w, y, rows, hidden, eps, stream, err, cap);
        if (nvec <= 64) return launch_warp_rows<T, 2>(x, w, y, rows, hidden, eps, stream, err, cap);
        return launch_warp_rows<T, 4>(x, w, y, rows, hidden, eps, stream, err, cap);
    }
    // Choose NV (vectors per thread) so the CTA has between 32 and 1024 threads.
    int nv = 0;
    if (vec_ok && variant != 2) {
        // Smallest NV giving <= 256 threads; NV = 8 stretches to 1024 threads (hidden <= 65536).
        for (int cand : {1, 2, 4, 8}) {
            const int64_t threads = (nvec + cand - 1) / cand;
            if (threads <= 256 || (cand == 8 && threads <= 1024)) {
                nv = cand;
                break;
            }
        }
    }
    const dim3 grid((unsigned)rows);
    if (nv > 0) {
        int64_t threads = (nvec + nv - 1) / nv;
        threads = ((threads + 31) / 32) * 32;
        const dim3 block((unsigned)threads);
        switch (nv) {
            case 1: rmsnorm_vec_kernel<T, 1><<<grid, block, 0, stream>>>(x, w, y, hidden, eps); break;
            case 2: rmsnorm_vec_kernel<T, 2><<<grid, block, 0, stream>>>(x, w, y, hidden, eps); break;
            case 4: rmsnorm_vec_kernel<T, 4><<<grid, block, 0, stream>>>(x, w, y, hidden, eps); break;
            default: rmsnorm_vec_kernel<T, 8><<<grid, block, 0, stream>>>(x, w, y, hidden, eps); break;
        }
    } else {
        rmsnorm_generic_kernel<T><<<grid, 256, 0, stream>>>(x, w, y, hidden, eps);
    }
    return sf::check_launch("rmsnorm launch", err, cap);
}

}  // namespace

// variant: 0 = dispatch by shape (vectorised when legal), 2 = force the general kernel.
int sf_rmsnorm_launch(const void* x, const void* w, void* y, int64_t rows, int64_t hidden, float eps,
                      int32_t dtype, int32_t variant, cudaStream_t stream, char* err, uint64_t cap) {
    if (rows < 0 || hidden < 1) return sf::fail(SF_EINVAL, err, cap, "rmsnorm: need rows >= 0 and hidden >= 1 (got %lld, %lld)", (long long)rows, (long long)hidden);
    if (!(eps > 0.f)) return sf::fail(SF_EINVAL, err, cap, "rmsnorm: eps must be > 0");
    if (rows == 0) return SF_OK;
    if (!x || !w || !y) return sf::fail(SF_EINVAL, err, cap, "rmsnorm: null tensor pointer");
    if (dtype == SF_DTYPE_F16)
        return launch_typed<__half>((const __half*)x, (const __half*)w, (__half*)y, rows, hidden, eps, variant, stream, err, cap);
    if (dtype == SF_DTYPE_BF16)
        return launch_typed<__nv_bfloat16>((const __nv_bfloat16*)x, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, rows, hidden,
                                           eps, variant, stream, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "rmsnorm: dtype %d is not fp16/bf16", dtype);
}

extern "C" int sf_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t hidden, float eps, int32_t dtype,
                          void* stream, char* err, uint64_t cap) {
    return sf_rmsnorm_launch(x, w, y, rows, hidden, eps, dtype, 0, (cudaStream_t)stream, err, cap);
}
