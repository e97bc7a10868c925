// gemv for sm_100a: y[r] = sum_k A[r, k] * x[k]     (tasks/gemv/reference.py, reference())
//
// A [M, K] row-major, x [K], y [M]; fp16 or bf16 in, fp32 accumulate, one rounding at the output.
// HBM-bound: A is read exactly once (2 bytes per multiply-add), x (K elements) is re-read by every
// row out of L1/L2.  One warp per row: each lane streams 16-byte vectors of its row, four of them
// in flight before the first multiply (64 bytes per lane, 2 KB per warp; with 8 resident 4-warp
// CTAs that is 64 KB in flight per SM, above the ~40 KB that HBM bandwidth x latency asks for),
// accumulates in fp32 and the warp reduces with shuffles; lane 0 stores y[r].  Rows are visited
// grid-stride by 4-warp CTAs, at most 8 per SM (64 registers per thread, no spills): 4096 rows are
// 1024 CTAs, one wave of 7 per SM, so the slowest SM reads at most one row more than the average.  Unaligned bases or K % 8 != 0 take the scalar loop (same order of
// operations per lane, element loads instead of vectors).  NaN/Inf in A or x propagate through the
// fp32 sums as in the fp64 reference.
#include "sf_common.cuh"

#include <algorithm>

namespace {

constexpr int WARPS = 4;
constexpr int UNROLL = 4;

// 16-byte load of x through L1 (x is shared by every row).
template <typename T>
__device__ __forceinline__ sf::Vec8<T> ld_x_v8(const T* p) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    sf::Vec8<T> out;
    *reinterpret_cast<uint4*>(&out) = raw;
    return out;
}

template <typename T>
__global__ void __launch_bounds__(WARPS * 32, 8) gemv_kernel(const T* __restrict__ A, const T* __restrict__ x, T* __restrict__ y,
                                                          int64_t M, int64_t K, bool vec) {
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (int64_t)blockIdx.x * WARPS + (threadIdx.x >> 5);
    const int64_t wstride = (int64_t)gridDim.x * WARPS;
    for (int64_t r = warp0; r < M; r += wstride) {
        const T* row = A + r * K;
        float acc0 = 0.f, acc1 = 0.f;
        if (vec) {
            const int64_t kv = K >> 3;
            for (int64_t v0 = lane; v0 < kv; v0 += 32 * UNROLL) {
                sf::Vec8<T> a[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    const int64_t v = v0 + 32 * u;
                    if (v < kv) a[u] = sf::ld_global_nc_v8<T>(row + v * 8);
                }
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    const int64_t v = v0 + 32 * u;
                    if (v < kv) {
                        const sf::Vec8<T> xv = ld_x_v8<T>(x + v * 8);
#pragma unroll
                        for (int j = 0; j < 8; j += 2) {
                            acc0 = fmaf(sf::Dt<T>::to_f(a[u].v[j]), sf::Dt<T>::to_f(xv.v[j]), acc0);
                            acc1 = fmaf(sf::Dt<T>::to_f(a[u].v[j + 1]), sf::Dt<T>::to_f(xv.v[j + 1]), acc1);
                        }
                    }
                }
            }
        } else {
            for (int64_t k = lane; k < K; k += 32) acc0 = fmaf(sf::Dt<T>::to_f(row[k]), sf::Dt<T>::to_f(x[k]), acc0);
        }
        float acc = acc0 + acc1;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        if (lane == 0) y[r] = sf::Dt<T>::from_f(acc);
    }
}

__global__ void zero_rows_kernel(uint16_t* __restrict__ y, int64_t m) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) y[i] = 0;
}

template <typename T>
int launch_t(const void* A, const void* x, void* y, int64_t M, int64_t K, int32_t variant, cudaStream_t s, char* err, uint64_t cap) {
    const bool vec = variant != 2 && (K % 8) == 0 && sf::aligned16(A) && sf::aligned16(x);
    int64_t blocks = (M + WARPS - 1) / WARPS;
    const int64_t cap_blocks = (int64_t)sf::sm_count() * 8;
    if (blocks > cap_blocks) blocks = cap_blocks;
    if (blocks < 1) blocks = 1;
    gemv_kernel<T><<<(unsigned)blocks, WARPS * 32, 0, s>>>((const T*)A, (const T*)x, (T*)y, M, K, vec);
    return sf::check_launch("gemv launch", err, cap);
}

}  // namespace

// variant 2 forces the scalar loop (any alignment); 0/1 take the vector loop when the bases are
// 16-byte aligned and K % 8 == 0.
int sf_gemv_launch(const void* A, const void* x, void* y, int64_t M, int64_t K, int32_t dtype, int32_t variant, cudaStream_t s,
                   char* err, uint64_t cap) {
    if (M < 0 || K < 0) return sf::fail(SF_EINVAL, err, cap, "gemv: negative size");
    if (dtype != SF_DTYPE_F16 && dtype != SF_DTYPE_BF16) return sf::fail(SF_EINVAL, err, cap, "gemv: dtype %d is not fp16/bf16", dtype);
    if (M == 0) return SF_OK;
    if (!y) return sf::fail(SF_EINVAL, err, cap, "gemv: null output pointer");
    if (K == 0) {
        // The empty sum: +0 in every row.
        zero_rows_kernel<<<(unsigned)std::min<int64_t>((M + 255) / 256, 1024), 256, 0, s>>>((uint16_t*)y, M);
        return sf::check_launch("gemv zero launch", err, cap);
    }
    if (!A || !x) return sf::fail(SF_EINVAL, err, cap, "gemv: null input pointer");
    if (dtype == SF_DTYPE_F16) return launch_t<__half>(A, x, y, M, K, variant, s, err, cap);
    return launch_t<__nv_bfloat16>(A, x, y, M, K, variant, s, err, cap);
}

extern "C" int sf_gemv(const void* A, const void* x, void* y, int64_t M, int64_t K, int32_t dtype, void* stream, char* err,
                       uint64_t cap) {
    return sf_gemv_launch(A, x, y, M, K, dtype, 0, (cudaStream_t)stream, err, cap);
}
