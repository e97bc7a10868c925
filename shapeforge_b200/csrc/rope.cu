// Rotate-half RoPE for sm_100a over x, y [B, H, S, D] (tasks/rope/reference.py:105-115):
//
//   half = D/2, inv_freq[i] = BASE^(-i/half), angle = s * inv_freq[i]
//   y[..., i]        = x[..., i] * cos(angle) - x[..., i+half] * sin(angle)
//   y[..., i + half] = x[..., i] * sin(angle) + x[..., i+half] * cos(angle)
//
// HBM-bound (2 x 16-bit per element in + out).  The angle depends only on (s, i), so a CTA owns a
// block of 32 positions and a share of the B*H heads: each thread issues the 16-byte x1/x2 loads of
// up to 8 heads of its share at once, computes the cos/sin of its 8 frequencies at its position
// while they are in flight (once per thread), then rotates and stores them.  inv_freq[i] = r^i with r = BASE^(-1/half) computed once on the
// host in double precision (a thread's first frequency by repeated squaring, the next ones by
// repeated multiplication: relative error below 2^-46); the angle s * inv_freq is formed and
// reduced modulo 2 pi in double precision, so positions in the thousands keep full accuracy, and
// the reduced angle (|a| <= pi) goes to the special-function sine/cosine (absolute error ~2^-21).
#include "sf_common.cuh"

#include <cmath>
#include <type_traits>

namespace {

constexpr int POS_PER_CTA = 32;

// Heads a thread handles per step: all their 16-byte loads are issued before the angles are
// computed, so the DRAM latency overlaps the double-precision angle reduction (4 for bf16, whose
// conversions need more registers, so that two CTAs still fit on an SM without spills).
template <typename T>
__host__ __device__ constexpr int heads_per_step() { return std::is_same<T, __half>::value ? 8 : 4; }

template <typename T>
__global__ void __launch_bounds__(256, 2) rope_vec_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t bh, int64_t S,
                                                       int64_t D, double ratio, int64_t bh_per_cta) {
    const int64_t half = D / 2;
    const int64_t vec_per_pos = half / 8;
    const int64_t local = threadIdx.x;
    const int64_t p = local / vec_per_pos;
    const int64_t iv = local % vec_per_pos;
    const int64_t s = (int64_t)blockIdx.x * POS_PER_CTA + p;
    if (p >= POS_PER_CTA || s >= S) return;
    const int64_t h0 = (int64_t)blockIdx.y * bh_per_cta;
    const int64_t h1 = min(bh, h0 + bh_per_cta);
    constexpr int HG = heads_per_step<T>();
    float c[8], sn[8];
    for (int64_t hb = h0; hb < h1; hb += HG) {
        sf::Vec8<T> a[HG], b[HG];
#pragma unroll
        for (int u = 0; u < HG; ++u) {
            if (hb + u < h1) {
                const T* xr = x + ((hb + u) * S + s) * D + iv * 8;
                a[u] = sf::ld_global_nc_v8<T>(xr);
                b[u] = sf::ld_global_nc_v8<T>(xr + half);
            }
        }
        if (hb == h0) {
            double f = 1.0, sq = ratio;
            for (int64_t e = iv * 8; e > 0; e >>= 1) {  // ratio^(8 iv)
                if (e & 1) f *= sq;
                sq *= sq;
            }
            constexpr double TWO_PI = 6.283185307179586476925286766559;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const double ang = (double)s * f;
                const double red = ang - rint(ang * (1.0 / TWO_PI)) * TWO_PI;
                __sincosf((float)red, &sn[j], &c[j]);
                f *= ratio;
            }
        }
#pragma unroll
        for (int u = 0; u < HG; ++u) {
            if (hb + u < h1) {
                sf::Vec8<T> o1, o2;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float x1 = sf::Dt<T>::to_f(a[u].v[j]), x2 = sf::Dt<T>::to_f(b[u].v[j]);
                    o1.v[j] = sf::Dt<T>::from_f(x1 * c[j] - x2 * sn[j]);
                    o2.v[j] = sf::Dt<T>::from_f(x1 * sn[j] + x2 * c[j]);
                }
                T* yr = y + ((hb + u) * S + s) * D + iv * 8;
                sf::st_global_v8<T>(yr, o1);
                sf::st_global_v8<T>(yr + half, o2);
            }
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(256) rope_generic_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t bh, int64_t S,
                                                           int64_t D, double base) {
    const int64_t half = D / 2;
    const int64_t total = bh * S * half;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t % half;
        const int64_t row = t / half;  // (h * S + s)
        const int64_t s = row % S;
        double sd, cd;
        sincos((double)s * pow(base, -(double)i / (double)half), &sd, &cd);
        const float c = (float)cd, sn = (float)sd;
        const float x1 = sf::Dt<T>::to_f(x[row * D + i]), x2 = sf::Dt<T>::to_f(x[row * D + half + i]);
        y[row * D + i] = sf::Dt<T>::from_f(x1 * c - x2 * sn);
        y[row * D + half + i] = sf::Dt<T>::from_f(x1 * sn + x2 * c);
    }
}

template <typename T>
int launch_t(const void* x, void* y, int64_t B, int64_t H, int64_t S, int64_t D, double base, int32_t variant, cudaStream_t st,
             char* err, uint64_t cap) {
    const int64_t bh = B * H;
    const int64_t half = D / 2;
    const bool vec = variant != 2 && half % 8 == 0 && sf::aligned16(x) && sf::aligned16(y) && (half / 8) * POS_PER_CTA <= 256;
    if (vec) {
        const int64_t pos_blocks = (S + POS_PER_CTA - 1) / POS_PER_CTA;
        // About two CTAs per SM in one wave; each walks a share of the heads, HG at a time.
        int64_t splits = (int64_t)sf::sm_count() * 2 / (pos_blocks > 0 ? pos_blocks : 1);
        if (splits < 1) splits = 1;
        if (splits > bh) splits = bh;
        if (splits > 65535) splits = 65535;
        const int64_t per = (bh + splits - 1) / splits;
        splits = (bh + per - 1) / per;
        if (pos_blocks > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "rope: S too large");
        const int threads = (int)((half / 8) * POS_PER_CTA);
        rope_vec_kernel<T><<<dim3((unsigned)pos_blocks, (unsigned)splits), threads, 0, st>>>((const T*)x, (T*)y, bh, S, D,
                                                                                             std::pow(base, -1.0 / (double)half), per);
    } else {
        const int64_t total = bh * S * half;
        int64_t blocks = (total + 255) / 256;
        const int64_t capb = (int64_t)sf::sm_count() * 16;
        if (blocks > capb) blocks = capb;
        if (blocks < 1) blocks = 1;
        rope_generic_kernel<T><<<(unsigned)blocks, 256, 0, st>>>((const T*)x, (T*)y, bh, S, D, base);
    }
    return sf::check_launch("rope launch", err, cap);
}

}  // namespace

int sf_rope_launch(const void* x, void* y, int64_t B, int64_t H, int64_t S, int64_t D, double base, int32_t dtype, int32_t variant,
                   cudaStream_t st, char* err, uint64_t cap) {
    if (B < 0 || H < 0 || S < 0 || D < 2 || D % 2) return sf::fail(SF_EINVAL, err, cap, "rope: need B,H,S >= 0 and an even D >= 2");
    if (!(base > 0)) return sf::fail(SF_EINVAL, err, cap, "rope: BASE must be > 0");
    if (B * H * S == 0) return SF_OK;
    if (!x || !y) return sf::fail(SF_EINVAL, err, cap, "rope: null tensor pointer");
    if (dtype == SF_DTYPE_F16) return launch_t<__half>(x, y, B, H, S, D, base, variant, st, err, cap);
    if (dtype == SF_DTYPE_BF16) return launch_t<__nv_bfloat16>(x, y, B, H, S, D, base, variant, st, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "rope: dtype %d is not fp16/bf16", dtype);
}

extern "C" int sf_rope(const void* x, void* y, int64_t B, int64_t H, int64_t S, int64_t D, double base, int32_t dtype, void* stream,
                       char* err, uint64_t cap) {
    return sf_rope_launch(x, y, B, H, S, D, base, dtype, 0, (cudaStream_t)stream, err, cap);
}
