// Shared-memory operand layouts and 16-bit helpers of the chunked gated-delta-rule kernels
// (kda_c32.cu, kda_split.cu).  All tiles use the 128-byte swizzle that the tcgen05 shared-memory
// descriptors of sm100.cuh describe.
#pragma once

#include "sf_common.cuh"

#include <stdint.h>

namespace kdal {

template <typename T>
__device__ __forceinline__ uint16_t to16(float x) {
    const T h = sf::Dt<T>::from_f(x);
    return *reinterpret_cast<const uint16_t*>(&h);
}
template <typename T>
__device__ __forceinline__ float from16(uint16_t u) {
    return sf::Dt<T>::to_f(*reinterpret_cast<const T*>(&u));
}

// Byte offset of fp32 element (row r, column c) of a K-major operand with the 128-byte swizzle,
// K-blocks of 32 columns `blk` bytes apart.
__device__ __forceinline__ int kmaj32(int r, int c, int blk) {
    return (c >> 5) * blk + r * 128 + ((((c & 31) >> 2) ^ (r & 7)) << 4) + ((c & 3) << 2);
}
// Byte offset of 16-bit element (row r = K index, column c = MN index) of an MN-major operand with
// the 128-byte swizzle, 64-column blocks `blk` bytes apart.
__device__ __forceinline__ int mnmaj16(int r, int c, int blk) {
    return (c >> 6) * blk + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + ((c & 7) << 1);
}
// Byte offset of the 16-byte chunk j (0..7) of row r in a 128-byte-swizzled row-major tile.
__device__ __forceinline__ int chunk128(int r, int j) { return r * 128 + (((j & 7) ^ (r & 7)) << 4); }

// e^x as one ex2.approx.ftz of x log2(e): the relative error is that of ex2.approx (about 2^-22)
// plus |x| times the rounding of x log2(e) (about 1e-5 at |x| = 80, the largest factor exponent);
// results below the fp32 normal range flush to zero, negligible against the other terms of the
// sums they enter.
__device__ __forceinline__ float fexp(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
    return y;
}

// Two fp32 values as packed 16-bit high parts (returned) and the 16-bit rounding of their
// residuals (`lo`); a non-finite high part gets a zero residual.
template <typename T>
__device__ __forceinline__ uint32_t pack_hi_lo(float x0, float x1, uint32_t& lo) {
    const uint16_t h0 = to16<T>(x0), h1 = to16<T>(x1);
    const float f0 = from16<T>(h0), f1 = from16<T>(h1);
    const float r0 = isfinite(f0) ? x0 - f0 : 0.f, r1 = isfinite(f1) ? x1 - f1 : 0.f;
    lo = (uint32_t)to16<T>(r0) | ((uint32_t)to16<T>(r1) << 16);
    return (uint32_t)h0 | ((uint32_t)h1 << 16);
}

// pack_hi_lo with packed conversions (one cvt for both high parts, one for both residuals).
template <typename T>
__device__ __forceinline__ uint32_t pack_hi_lo2(float x0, float x1, uint32_t& lo);

template <>
__device__ __forceinline__ uint32_t pack_hi_lo2<__nv_bfloat16>(float x0, float x1, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float2 f = __bfloat1622float2(h);
    const float r0 = fabsf(f.x) < INFINITY ? x0 - f.x : 0.f, r1 = fabsf(f.y) < INFINITY ? x1 - f.y : 0.f;
    const __nv_bfloat162 l = __floats2bfloat162_rn(r0, r1);
    lo = *reinterpret_cast<const uint32_t*>(&l);
    return *reinterpret_cast<const uint32_t*>(&h);
}

template <>
__device__ __forceinline__ uint32_t pack_hi_lo2<__half>(float x0, float x1, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 f = __half22float2(h);
    const float r0 = fabsf(f.x) < INFINITY ? x0 - f.x : 0.f, r1 = fabsf(f.y) < INFINITY ? x1 - f.y : 0.f;
    const __half2 l = __floats2half2_rn(r0, r1);
    lo = *reinterpret_cast<const uint32_t*>(&l);
    return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace kdal
