// Flash-attention forward on the tcgen05 tensor cores, sm_100a.
//
//   o[b,h,i,:] = sum_j softmax_j(q[b,h,i,:] . k[b,h,j,:] * scale [+ causal mask j <= i]) v[b,h,j,:]
//
// Task contract: tasks/flash_attention/reference.py:113-119 (non-causal scaled_dot_product_attention
// in fp32, SM_SCALE attr); the causal workload is the same formula with the mask.  q, k, v, o are
// [B, H, S, D] row-major fp16/bf16, D in {64, 128}; softmax statistics in fp32.
//
// One CTA per (b*h, 128-query tile), two CTAs resident per SM (256 TMEM columns, ~97 KB of shared
// memory each), so one CTA's softmax, prologue and epilogue overlap the other's MMAs; 192 threads:
//   warp 0      TMA producer: Q once, then K_j and V_j tiles of 128 keys into their own slots
//               (one slot each for D=128, two for D=64; 3-D tensor maps over [B*H, S, D], so rows
//               past S read as zeros and never spill into the next head);
//   warp 1      MMA issuer: S_j = Q.K_j^T (M=128, N=128, K=D) into TMEM columns [0,128), then, once
//               the softmax has written P_j over those columns, O += P_j.V_j (M=128, N=D, K=128)
//               with P read from TMEM as the A operand and V as an MN-major operand straight from
//               its [keys, D] layout.  S_{j+1} is issued after P_j.V_j into the same columns: the
//               tensor pipe executes one CTA's MMAs in issue order, so P_j is read before it is
//               overwritten, and the commit that publishes S_{j+1} also covers P_j.V_j;
//   warps 2..5  softmax, one thread per query row: two passes over the score row in TMEM (row max,
//               then exp2 and P), online max/sum in fp32; O is rescaled in TMEM (tcgen05.ld/st) only
//               when the row max grows by more than 2^8 (the final 1/l cancels any stale max, so this
//               is exact up to rounding); P_j is written as a 16-bit high part and a 16-bit residual
//               into the score columns it was computed from.  Final O / l is stored with 16-byte
//               stores.
// Causal CTAs skip every key tile above the diagonal.  Blocks walk groups of heads whose K/V fit
// in L2 together, heaviest query tiles first within a group.
// NaN/Inf follow the fp32 reference: the row max propagates NaN, so a special in a query row makes
// that output row NaN.  Every mbarrier wait is bounded.
#include "sf_common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <cudaTypedefs.h>
#include <algorithm>
#include <mutex>
#include <type_traits>

__device__ sm100::KernelStatus g_attn_status;

namespace {

constexpr int BM = 128, BN = 128;
constexpr int BOX_BYTES = 128 * 128;  // 128 rows x 64 16-bit elements
constexpr int NUM_THREADS = 192;
constexpr uint32_t TMEM_COLS = 256;   // S_j / P_j [0,128), O [128, 128 + D)
constexpr uint32_t O_COL = 128;

struct __align__(8) Bars {
    uint64_t q_full;
    uint64_t k_full[2], k_empty[2];
    uint64_t v_full[2], v_empty[2];
    uint64_t s_full;
    uint64_t p_full[2];  // keys [0,64) and [64,128) of P_j written
    uint64_t o_done;
    uint32_t tmem_base;
};

__device__ __forceinline__ float nan_max(float a, float b) { return (b > a || b != b) ? b : a; }

// max that returns NaN if either operand is NaN (one instruction).
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

// 2^x on the special-function unit (approximate, subnormal results flushed to zero; softmax
// weights below 2^-126 of the row max contribute nothing at fp32 accumulation).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max of three that returns NaN if any operand is NaN (one instruction on sm_100).
__device__ __forceinline__ float fmax3_nan(float a, float b, float c) {
    float d;
    asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Packed fp32 pair arithmetic (one FFMA2 / FADD2 for two lanes of work).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(reinterpret_cast<uint64_t&>(d))
        : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)), "l"(reinterpret_cast<const uint64_t&>(c)));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("add.rn.f32x2 %0, %1, %2;"
        : "=l"(reinterpret_cast<uint64_t&>(d))
        : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)));
    return d;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// P is written as a 16-bit high part and a 16-bit residual (P - high), and P.V is issued twice, so
// the probabilities enter the product with ~16-22 significant bits instead of 8-11: a single
// 16-bit rounding of P, amplified by cancellation between large v terms, exceeds the task
// tolerances.  Keys [32q, 32q + 32) of a tile go to TMEM columns [32q, 32q + 16) (high, two keys
// per column) and [32q + 16, 32q + 32) (residual): each quarter overwrites only the score columns
// it was computed from.
__device__ __forceinline__ uint32_t p_hi_col(int kk) { return (uint32_t)(32 * (kk >> 1) + 8 * (kk & 1)); }
__device__ __forceinline__ uint32_t p_lo_col(int kk) { return p_hi_col(kk) + 16u; }

template <int D>
struct Layout {
    static constexpr int DB = D / 64;                  // 64-column boxes per row
    static constexpr int NST = D == 64 ? 2 : 1;        // K (and V) slots
    static constexpr int TILE = DB * BOX_BYTES;        // one 128-row tile
    static constexpr int Q = 0;
    static constexpr int K = Q + TILE;                 // K[NST]
    static constexpr int V = K + NST * TILE;           // V[NST]
    static constexpr int BARS = V + NST * TILE;
    static constexpr int BYTES = BARS + 256;
};

// One score tile of one query row (the calling thread's TMEM lane): row max, lazy rescale of O,
// exponentials, P_j (high + residual) over the score columns, published a half at a time on
// p_full[0] / p_full[1].  MASK: keys past `lim` (tile-relative) score -inf.  `o_ready` (when not
// null) completes a phase per P.V: a warp that must rescale O first waits for P_{j-1}.V_{j-1}
// (the kernel that double-buffers S issues S_{j+1} before P_j.V_j, so S_j does not imply it).
template <typename T, int D, bool MASK>
__device__ __forceinline__ void softmax_tile(uint32_t tmem, uint32_t tmem_o, uint32_t lane_off, int lim, int j, float scale_log2,
                                             float& m, float& l, uint64_t* p_full, uint64_t* o_ready = nullptr,
                                             sm100::KernelStatus* status = nullptr) {
    constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
    // Pass 1: row max of the raw scores (scale > 0 commutes with max); NaN propagates.
    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t r[64];
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)(64 * h), *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)(64 * h + 32), *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        sm100::tmem_ld_wait();
        if (MASK) {
#pragma unroll
            for (int c = 0; c < 64; ++c)
                if (64 * h + c > lim) r[c] = 0xff800000u;  // -inf
        }
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
            const float a = fmax3_nan(__uint_as_float(r[c]), __uint_as_float(r[c + 1]), __uint_as_float(r[c + 2]));
            const float b = fmax3_nan(__uint_as_float(r[c + 3]), __uint_as_float(r[c + 4]), __uint_as_float(r[c + 5]));
            const int k = (c >> 3) & 3;
            mx[k] = fmax3_nan(mx[k], a, fmax3_nan(b, __uint_as_float(r[c + 6]), __uint_as_float(r[c + 7])));
        }
    }
    const float rmax = fmax3_nan(mx[0], mx[1], fmax_nan(mx[2], mx[3]));
    const float m_new = fmax_nan(m, rmax * scale_log2);
    const bool need = !(m_new <= m + 8.0f);
    const float m_old = m;
    if (need) m = m_new;
    // P.V_{j-1} has completed: the commit that published S_j was issued after it (or, with
    // o_ready, once that barrier's phase j - 1 is complete).
    if (j > 0) {
        const float alpha = need ? ex2_approx(m_old - m_new) : 1.0f;
        if (__any_sync(0xffffffffu, need)) {
            if (o_ready) {
                sm100::mbar_wait(o_ready, (uint32_t)(j - 1) & 1u, status, 40);
                sm100::tc_fence_after();
            }
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem_o + lane_off + (uint32_t)(c * 32), r);
                sm100::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                sm100::tmem_st_32x32b_x32(tmem_o + lane_off + (uint32_t)(c * 32), r);
            }
        }
        if (need) l *= alpha;
    }
    // Pass 2: p = 2^(s * scale * log2(e) - m), one FFMA2 per two scores and one MUFU.EX2 per score;
    // P over the score columns just read, a quarter of the keys at a time; each half of the keys is
    // published as soon as it is in TMEM.
    const float2 sc2 = make_float2(scale_log2, scale_log2);
    const float2 nm2 = make_float2(-m, -m);
    const float2 neg1 = make_float2(-1.f, -1.f);
    float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
        uint32_t r[64];
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)(64 * h), *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)(64 * h + 32), *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        sm100::tmem_ld_wait();
        if (MASK) {
#pragma unroll
            for (int c = 0; c < 64; ++c)
                if (64 * h + c > lim) r[c] = 0xff800000u;
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            uint32_t hv[16], lv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float2 x = ffma2(make_float2(__uint_as_float(r[32 * e + 2 * i]), __uint_as_float(r[32 * e + 2 * i + 1])), sc2, nm2);
                const float2 pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                acc[i & 3] = fadd2(acc[i & 3], pp);
                if (BF16) {
                    // bf16: the high part is the upper half of the fp32 bits (truncation, one byte
                    // permute for two values) and the residual p - high is exact in fp32, so only the
                    // residual is rounded: ~16 significant bits in total.
                    const uint32_t b0 = __float_as_uint(pp.x), b1 = __float_as_uint(pp.y);
                    hv[i] = __byte_perm(b0, b1, 0x7632);
                    const float2 res = ffma2(make_float2(__uint_as_float(b0 & 0xFFFF0000u), __uint_as_float(b1 & 0xFFFF0000u)), neg1, pp);
                    lv[i] = pack2<T>(res.x, res.y);
                } else {
                    hv[i] = pack2<T>(pp.x, pp.y);
                    const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hv[i]));
                    const float2 res = ffma2(hf, neg1, pp);
                    lv[i] = pack2<T>(res.x, res.y);
                }
            }
            const uint32_t col = (uint32_t)(64 * h + 32 * e);
            sm100::tmem_st_32x32b_x16(tmem + lane_off + col, hv);
            sm100::tmem_st_32x32b_x16(tmem + lane_off + col + 16u, lv);
        }
        sm100::tmem_st_wait();
        sm100::tc_fence_before();
        sm100::mbar_arrive(&p_full[h]);
    }
    const float2 t = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
    l += t.x + t.y;
}

// softmax_tile with keys [64, 128) kept in registers between the two passes and that half of P
// published first (one TMEM reload of keys [0, 64) instead of two of all keys); it needs ~64 more
// registers, which the two-CTA kernel's bf16 instantiations do not have without spilling.
// One score tile of one query row (the calling thread's TMEM lane): row max, lazy rescale of O,
// exponentials, P_j (high + residual) over the score columns, published a half at a time on
// p_full[0] / p_full[1].  MASK: keys past `lim` (tile-relative) score -inf.  `o_ready` (when not
// null) completes a phase per P.V: a warp that must rescale O first waits for P_{j-1}.V_{j-1}
// (the kernel that double-buffers S issues S_{j+1} before P_j.V_j, so S_j does not imply it).
template <typename T, int D, bool MASK>
__device__ __forceinline__ void softmax_tile_kh(uint32_t tmem, uint32_t tmem_o, uint32_t lane_off, int lim, int j, float scale_log2,
                                             float& m, float& l, uint64_t* p_full, uint64_t* o_ready = nullptr,
                                             sm100::KernelStatus* status = nullptr) {
    constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
    // Pass 1: row max of the raw scores (scale > 0 commutes with max); NaN propagates.  Keys
    // [64, 128) stay in registers (rb) for pass 2, which writes that half of P first; keys [0, 64)
    // are read again.
    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    uint32_t rb[64];
    {
        uint32_t r[64];
        sm100::tmem_ld_32x32b_x32(tmem + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + 32u, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + 64u, *reinterpret_cast<uint32_t(*)[32]>(&rb[0]));
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + 96u, *reinterpret_cast<uint32_t(*)[32]>(&rb[32]));
        sm100::tmem_ld_wait();
        if (MASK) {
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                if (c > lim) r[c] = 0xff800000u;  // -inf
                if (64 + c > lim) rb[c] = 0xff800000u;
            }
        }
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
            const float a = fmax3_nan(__uint_as_float(r[c]), __uint_as_float(r[c + 1]), __uint_as_float(r[c + 2]));
            const float b = fmax3_nan(__uint_as_float(r[c + 3]), __uint_as_float(r[c + 4]), __uint_as_float(r[c + 5]));
            const int k = (c >> 3) & 3;
            mx[k] = fmax3_nan(mx[k], a, fmax3_nan(b, __uint_as_float(r[c + 6]), __uint_as_float(r[c + 7])));
        }
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
            const float a = fmax3_nan(__uint_as_float(rb[c]), __uint_as_float(rb[c + 1]), __uint_as_float(rb[c + 2]));
            const float b = fmax3_nan(__uint_as_float(rb[c + 3]), __uint_as_float(rb[c + 4]), __uint_as_float(rb[c + 5]));
            const int k = (c >> 3) & 3;
            mx[k] = fmax3_nan(mx[k], a, fmax3_nan(b, __uint_as_float(rb[c + 6]), __uint_as_float(rb[c + 7])));
        }
    }
    const float rmax = fmax3_nan(mx[0], mx[1], fmax_nan(mx[2], mx[3]));
    const float m_new = fmax_nan(m, rmax * scale_log2);
    const bool need = !(m_new <= m + 8.0f);
    const float m_old = m;
    if (need) m = m_new;
    // P.V_{j-1} has completed: the commit that published S_j was issued after it (or, with
    // o_ready, once that barrier's phase j - 1 is complete).
    if (j > 0) {
        const float alpha = need ? ex2_approx(m_old - m_new) : 1.0f;
        if (__any_sync(0xffffffffu, need)) {
            if (o_ready) {
                sm100::mbar_wait(o_ready, (uint32_t)(j - 1) & 1u, status, 40);
                sm100::tc_fence_after();
            }
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem_o + lane_off + (uint32_t)(c * 32), r);
                sm100::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
                sm100::tmem_st_32x32b_x32(tmem_o + lane_off + (uint32_t)(c * 32), r);
            }
        }
        if (need) l *= alpha;
    }
    // Pass 2: p = 2^(s * scale * log2(e) - m), one FFMA2 per two scores and one MUFU.EX2 per score;
    // P over the score columns just read, a quarter of the keys at a time; each half of the keys is
    // published as soon as it is in TMEM (keys [64, 128) first, from registers).
    const float2 sc2 = make_float2(scale_log2, scale_log2);
    const float2 nm2 = make_float2(-m, -m);
    const float2 neg1 = make_float2(-1.f, -1.f);
    float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
    auto half_p = [&](const uint32_t (&r)[64], int h) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            uint32_t hv[16], lv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float2 x = ffma2(make_float2(__uint_as_float(r[32 * e + 2 * i]), __uint_as_float(r[32 * e + 2 * i + 1])), sc2, nm2);
                const float2 pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
                acc[i & 3] = fadd2(acc[i & 3], pp);
                if (BF16) {
                    // bf16: the high part is the upper half of the fp32 bits (truncation, one byte
                    // permute for two values) and the residual p - high is exact in fp32, so only the
                    // residual is rounded: ~16 significant bits in total.
                    const uint32_t b0 = __float_as_uint(pp.x), b1 = __float_as_uint(pp.y);
                    hv[i] = __byte_perm(b0, b1, 0x7632);
                    const float2 res = ffma2(make_float2(__uint_as_float(b0 & 0xFFFF0000u), __uint_as_float(b1 & 0xFFFF0000u)), neg1, pp);
                    lv[i] = pack2<T>(res.x, res.y);
                } else {
                    hv[i] = pack2<T>(pp.x, pp.y);
                    const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hv[i]));
                    const float2 res = ffma2(hf, neg1, pp);
                    lv[i] = pack2<T>(res.x, res.y);
                }
            }
            const uint32_t col = (uint32_t)(64 * h + 32 * e);
            sm100::tmem_st_32x32b_x16(tmem + lane_off + col, hv);
            sm100::tmem_st_32x32b_x16(tmem + lane_off + col + 16u, lv);
        }
        sm100::tmem_st_wait();
        sm100::tc_fence_before();
        sm100::mbar_arrive(&p_full[h]);
    };
    half_p(rb, 1);
    {
        uint32_t r[64];
        sm100::tmem_ld_32x32b_x32(tmem + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + 32u, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        sm100::tmem_ld_wait();
        if (MASK) {
#pragma unroll
            for (int c = 0; c < 64; ++c)
                if (c > lim) r[c] = 0xff800000u;
        }
        half_p(r, 0);
    }
    const float2 t = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
    l += t.x + t.y;
}

template <typename T, int D, bool CAUSAL>
__global__ void __launch_bounds__(NUM_THREADS, 2)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                  T* __restrict__ o, int S, int BH, int nq, int group, float scale_log2, sm100::KernelStatus* status) {
    using L = Layout<D>;
    constexpr int DB = L::DB;
    constexpr int NST = L::NST;
    constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr bool KH = !BF16;  // keys [64, 128) kept in registers between the softmax passes
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + L::BARS);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Block -> (head, query tile): groups of `group` heads, heaviest query tiles first in a group.
    const int64_t per_group = (int64_t)group * nq;
    const int g = (int)((int64_t)blockIdx.x / per_group);
    const int hbase = g * group;
    const int gsize = min(group, BH - hbase);
    const int rem = (int)((int64_t)blockIdx.x - (int64_t)g * per_group);
    const int bh = hbase + rem % gsize;
    const int qt = CAUSAL ? (nq - 1 - rem / gsize) : rem / gsize;
    const int nkv_all = (S + BN - 1) / BN;
    const int nkv = CAUSAL ? min(qt + 1, nkv_all) : nkv_all;

    if (threadIdx.x == 0) {
        sm100::mbar_init(&bars->q_full, 1);
        for (int i = 0; i < NST; ++i) {
            sm100::mbar_init(&bars->k_full[i], 1);
            sm100::mbar_init(&bars->k_empty[i], 1);
            sm100::mbar_init(&bars->v_full[i], 1);
            sm100::mbar_init(&bars->v_empty[i], 1);
        }
        sm100::mbar_init(&bars->s_full, 1);
        sm100::mbar_init(&bars->p_full[0], 128);
        sm100::mbar_init(&bars->p_full[1], 128);
        sm100::mbar_init(&bars->o_done, 1);
        sm100::fence_mbar_init();
    }
    if (warp == 1) {
        sm100::tmem_alloc(&bars->tmem_base, TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    const uint32_t tmem_o = tmem + O_COL;

    if (warp == 0) {
        if (lane == 0) {
            sm100::tma_prefetch_desc(&tq);
            sm100::tma_prefetch_desc(&tk);
            sm100::tma_prefetch_desc(&tv);
            sm100::mbar_arrive_expect_tx(&bars->q_full, L::TILE);
            for (int b = 0; b < DB; ++b) sm100::tma_load_3d(smem + L::Q + b * BOX_BYTES, &tq, &bars->q_full, b * 64, qt * BM, bh);
            for (int j = 0; j < nkv; ++j) {
                const int st = j % NST;
                const uint32_t ph = (uint32_t)(j / NST) & 1u;
                if (!sm100::mbar_wait(&bars->k_empty[st], ph ^ 1u, status, 31)) break;
                sm100::mbar_arrive_expect_tx(&bars->k_full[st], L::TILE);
                for (int b = 0; b < DB; ++b)
                    sm100::tma_load_3d(smem + L::K + st * L::TILE + b * BOX_BYTES, &tk, &bars->k_full[st], b * 64, j * BN, bh);
                if (!sm100::mbar_wait(&bars->v_empty[st], ph ^ 1u, status, 32)) break;
                sm100::mbar_arrive_expect_tx(&bars->v_full[st], L::TILE);
                for (int b = 0; b < DB; ++b)
                    sm100::tma_load_3d(smem + L::V + st * L::TILE + b * BOX_BYTES, &tv, &bars->v_full[st], b * 64, j * BN, bh);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = sm100::idesc_f16(BM, BN, BF16);
            constexpr uint32_t idesc_o = sm100::idesc_f16_bmn(BM, D, BF16);
            const uint32_t sq = sm100::smem_u32(smem + L::Q);
            bool ok = sm100::mbar_wait(&bars->q_full, 0, status, 33);
            for (int j = 0; j < nkv && ok; ++j) {
                const int st = j % NST;
                const uint32_t ph = (uint32_t)(j / NST) & 1u;
                // S_j = Q . K_j^T into columns [0, 128).  Issued after P_{j-1}.V_{j-1}, which read
                // the same columns: the pipe runs this CTA's MMAs in issue order.
                if (!sm100::mbar_wait(&bars->k_full[st], ph, status, 34)) {
                    ok = false;
                    break;
                }
                sm100::tc_fence_after();
                const uint32_t sk = sm100::smem_u32(smem + L::K + st * L::TILE);
#pragma unroll
                for (int k = 0; k < D / 16; ++k) {
                    const uint32_t off = (uint32_t)((k >> 2) * BOX_BYTES + (k & 3) * 32);
                    sm100::mma_f16(tmem, sm100::smem_desc_k_sw128(sq + off), sm100::smem_desc_k_sw128(sk + off), idesc_s, k > 0 ? 1u : 0u);
                }
                sm100::mma_commit(&bars->s_full);
                sm100::mma_commit(&bars->k_empty[st]);
                // O += P_j . V_j, each half of the keys as soon as the softmax has written its P
                // (high part, then the residual).
                if (!sm100::mbar_wait(&bars->v_full[st], ph, status, 36)) {
                    ok = false;
                    break;
                }
                const uint32_t sv = sm100::smem_u32(smem + L::V + st * L::TILE);
                // The half of P the softmax publishes first: keys [64, 128) with softmax_tile_kh
                // (fp16), keys [0, 64) with softmax_tile (bf16, whose registers do not allow it).
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int half = KH ? 1 - hh : hh;
                    if (!sm100::mbar_wait(&bars->p_full[half], (uint32_t)j & 1u, status, 35)) {
                        ok = false;
                        break;
                    }
                    sm100::tc_fence_after();
#pragma unroll
                    for (int kk = 4 * half; kk < 4 * half + 4; ++kk) {
                        const uint64_t bd = sm100::smem_desc_mn_sw128(sv + (uint32_t)(kk * 16 * 128), BOX_BYTES, 1024);
                        sm100::mma_f16_ta(tmem_o, tmem + p_hi_col(kk), bd, idesc_o, (j > 0 || hh > 0 || kk > 4 * half) ? 1u : 0u);
                    }
#pragma unroll
                    for (int kk = 4 * half; kk < 4 * half + 4; ++kk) {
                        const uint64_t bd = sm100::smem_desc_mn_sw128(sv + (uint32_t)(kk * 16 * 128), BOX_BYTES, 1024);
                        sm100::mma_f16_ta(tmem_o, tmem + p_lo_col(kk), bd, idesc_o, 1u);
                    }
                }
                if (!ok) break;
                sm100::mma_commit(&bars->v_empty[st]);
            }
            if (ok) sm100::mma_commit(&bars->o_done);
        }
    } else {
        // ---------------- softmax: one thread per query row ----------------
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const int q = qt * BM + row;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            if (!sm100::mbar_wait(&bars->s_full, (uint32_t)j & 1u, status, 37)) {
                ok = false;
                break;
            }
            sm100::tc_fence_after();
            // Only the diagonal tile (causal) and the last tile (S tail) need a mask.
            const int key0 = j * BN;
            const bool masked = (CAUSAL && j == qt) || key0 + BN > S;
            const int lim = masked ? min(CAUSAL && j == qt ? row : BN - 1, S - 1 - key0) : BN - 1;
            if (KH) {
                if (masked)
                    softmax_tile_kh<T, D, true>(tmem, tmem_o, lane_off, lim, j, scale_log2, m, l, &bars->p_full[0]);
                else
                    softmax_tile_kh<T, D, false>(tmem, tmem_o, lane_off, lim, j, scale_log2, m, l, &bars->p_full[0]);
            } else {
                if (masked)
                    softmax_tile<T, D, true>(tmem, tmem_o, lane_off, lim, j, scale_log2, m, l, &bars->p_full[0]);
                else
                    softmax_tile<T, D, false>(tmem, tmem_o, lane_off, lim, j, scale_log2, m, l, &bars->p_full[0]);
            }
        }
        // ---------------- epilogue: O / l ----------------
        if (ok && nkv > 0 && sm100::mbar_wait(&bars->o_done, 0, status, 39)) {
            sm100::tc_fence_after();
            const float inv = 1.0f / l;
            T* orow = o + ((int64_t)bh * S + q) * D;
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem_o + lane_off + (uint32_t)(c * 32), r);
                sm100::tmem_ld_wait();
                if (q < S) {
                    uint4* d4 = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        d4[i] = make_uint4(pack2<T>(__uint_as_float(r[8 * i + 0]) * inv, __uint_as_float(r[8 * i + 1]) * inv),
                                           pack2<T>(__uint_as_float(r[8 * i + 2]) * inv, __uint_as_float(r[8 * i + 3]) * inv),
                                           pack2<T>(__uint_as_float(r[8 * i + 4]) * inv, __uint_as_float(r[8 * i + 5]) * inv),
                                           pack2<T>(__uint_as_float(r[8 * i + 6]) * inv, __uint_as_float(r[8 * i + 7]) * inv));
                }
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 1) sm100::tmem_dealloc(tmem, TMEM_COLS);
}

// ---- small grids: one CTA per SM, S double-buffered -----------------------------------------------
// When the (b*h, query tile) grid is at most one CTA per SM, no second CTA shares an SM to run its
// MMAs under this CTA's softmax, so this kernel overlaps them inside the CTA: 512 TMEM columns,
// S_j in [128 (j & 1), 128 (j & 1) + 128), O in [256, 256 + D).  The MMA warp issues S_0, S_1,
// P_0.V_0, S_2, P_1.V_1, ...: S_{j+1} runs on the tensor pipe while the softmax works on S_j, and
// S_{j+2} is issued after P_j.V_j, which read the same columns (the pipe runs one CTA's MMAs in
// issue order).  K and V have NST slots each.  (On full grids two CTAs per SM of fa_fwd_kernel are
// faster: 693 against 619 TF/s at causal B4 H32 S2048 D128.)
constexpr uint32_t DB_TMEM_COLS = 512;
constexpr uint32_t DB_O_COL = 256;

template <int D>
struct LayoutDB {
    static constexpr int DB = D / 64;
    static constexpr int NST = D == 64 ? 4 : 2;
    static constexpr int TILE = DB * BOX_BYTES;
    static constexpr int Q = 0;
    static constexpr int K = Q + TILE;
    static constexpr int V = K + NST * TILE;
    static constexpr int BARS = V + NST * TILE;
    static constexpr int BYTES = BARS + 512;
};

struct __align__(8) BarsDB {
    uint64_t q_full;
    uint64_t k_full[4], k_empty[4];
    uint64_t v_full[4], v_empty[4];
    uint64_t s_full[2];      // S buffer b holds S_j (j & 1 == b); one phase per use
    uint64_t p_full[2][2];   // P_j of buffer b, keys [0,64) and [64,128)
    uint64_t o_ready;        // one phase per P_j.V_j
    uint64_t o_done;
    uint32_t tmem_base;
};

template <typename T, int D, bool CAUSAL>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    fa_fwd_db_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                     T* __restrict__ o, int S, int BH, int nq, int group, float scale_log2, sm100::KernelStatus* status) {
    using L = LayoutDB<D>;
    constexpr int DB = L::DB;
    constexpr int NST = L::NST;
    constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    BarsDB* bars = reinterpret_cast<BarsDB*>(smem + L::BARS);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t per_group = (int64_t)group * nq;
    const int g = (int)((int64_t)blockIdx.x / per_group);
    const int hbase = g * group;
    const int gsize = min(group, BH - hbase);
    const int rem = (int)((int64_t)blockIdx.x - (int64_t)g * per_group);
    const int bh = hbase + rem % gsize;
    const int qt = CAUSAL ? (nq - 1 - rem / gsize) : rem / gsize;
    const int nkv_all = (S + BN - 1) / BN;
    const int nkv = CAUSAL ? min(qt + 1, nkv_all) : nkv_all;

    if (threadIdx.x == 0) {
        sm100::mbar_init(&bars->q_full, 1);
        for (int i = 0; i < NST; ++i) {
            sm100::mbar_init(&bars->k_full[i], 1);
            sm100::mbar_init(&bars->k_empty[i], 1);
            sm100::mbar_init(&bars->v_full[i], 1);
            sm100::mbar_init(&bars->v_empty[i], 1);
        }
        for (int b = 0; b < 2; ++b) {
            sm100::mbar_init(&bars->s_full[b], 1);
            sm100::mbar_init(&bars->p_full[b][0], 128);
            sm100::mbar_init(&bars->p_full[b][1], 128);
        }
        sm100::mbar_init(&bars->o_ready, 1);
        sm100::mbar_init(&bars->o_done, 1);
        sm100::fence_mbar_init();
    }
    if (warp == 1) {
        sm100::tmem_alloc(&bars->tmem_base, DB_TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    const uint32_t tmem_o = tmem + DB_O_COL;

    if (warp == 0) {
        if (lane == 0) {
            sm100::tma_prefetch_desc(&tq);
            sm100::tma_prefetch_desc(&tk);
            sm100::tma_prefetch_desc(&tv);
            sm100::mbar_arrive_expect_tx(&bars->q_full, L::TILE);
            for (int b = 0; b < DB; ++b) sm100::tma_load_3d(smem + L::Q + b * BOX_BYTES, &tq, &bars->q_full, b * 64, qt * BM, bh);
            for (int j = 0; j < nkv; ++j) {
                const int st = j % NST;
                const uint32_t ph = (uint32_t)(j / NST) & 1u;
                if (!sm100::mbar_wait(&bars->k_empty[st], ph ^ 1u, status, 41)) break;
                sm100::mbar_arrive_expect_tx(&bars->k_full[st], L::TILE);
                for (int b = 0; b < DB; ++b)
                    sm100::tma_load_3d(smem + L::K + st * L::TILE + b * BOX_BYTES, &tk, &bars->k_full[st], b * 64, j * BN, bh);
                if (!sm100::mbar_wait(&bars->v_empty[st], ph ^ 1u, status, 42)) break;
                sm100::mbar_arrive_expect_tx(&bars->v_full[st], L::TILE);
                for (int b = 0; b < DB; ++b)
                    sm100::tma_load_3d(smem + L::V + st * L::TILE + b * BOX_BYTES, &tv, &bars->v_full[st], b * 64, j * BN, bh);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = sm100::idesc_f16(BM, BN, BF16);
            constexpr uint32_t idesc_o = sm100::idesc_f16_bmn(BM, D, BF16);
            const uint32_t sq = sm100::smem_u32(smem + L::Q);
            bool ok = sm100::mbar_wait(&bars->q_full, 0, status, 43);
            // S_j = Q . K_j^T into buffer j & 1.
            auto issue_s = [&](int j) -> bool {
                const int st = j % NST;
                if (!sm100::mbar_wait(&bars->k_full[st], (uint32_t)(j / NST) & 1u, status, 44)) return false;
                sm100::tc_fence_after();
                const uint32_t sk = sm100::smem_u32(smem + L::K + st * L::TILE);
                const uint32_t dst = tmem + 128u * (uint32_t)(j & 1);
#pragma unroll
                for (int k = 0; k < D / 16; ++k) {
                    const uint32_t off = (uint32_t)((k >> 2) * BOX_BYTES + (k & 3) * 32);
                    sm100::mma_f16(dst, sm100::smem_desc_k_sw128(sq + off), sm100::smem_desc_k_sw128(sk + off), idesc_s, k > 0 ? 1u : 0u);
                }
                sm100::mma_commit(&bars->s_full[j & 1]);
                sm100::mma_commit(&bars->k_empty[st]);
                return true;
            };
            if (ok && nkv > 0) ok = issue_s(0);
            for (int j = 0; j < nkv && ok; ++j) {
                if (j + 1 < nkv && !issue_s(j + 1)) {
                    ok = false;
                    break;
                }
                // O += P_j . V_j, each half of the keys as soon as the softmax has written its P.
                const int st = j % NST;
                if (!sm100::mbar_wait(&bars->v_full[st], (uint32_t)(j / NST) & 1u, status, 46)) {
                    ok = false;
                    break;
                }
                const uint32_t sv = sm100::smem_u32(smem + L::V + st * L::TILE);
                const uint32_t pb = tmem + 128u * (uint32_t)(j & 1);
                // Keys [64, 128) first: the softmax publishes that half of P first.
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int half = 1 - hh;
                    if (!sm100::mbar_wait(&bars->p_full[j & 1][half], (uint32_t)(j >> 1) & 1u, status, 45)) {
                        ok = false;
                        break;
                    }
                    sm100::tc_fence_after();
#pragma unroll
                    for (int kk = 4 * half; kk < 4 * half + 4; ++kk) {
                        const uint64_t bd = sm100::smem_desc_mn_sw128(sv + (uint32_t)(kk * 16 * 128), BOX_BYTES, 1024);
                        sm100::mma_f16_ta(tmem_o, pb + p_hi_col(kk), bd, idesc_o, (j > 0 || hh > 0 || kk > 4) ? 1u : 0u);
                    }
#pragma unroll
                    for (int kk = 4 * half; kk < 4 * half + 4; ++kk) {
                        const uint64_t bd = sm100::smem_desc_mn_sw128(sv + (uint32_t)(kk * 16 * 128), BOX_BYTES, 1024);
                        sm100::mma_f16_ta(tmem_o, pb + p_lo_col(kk), bd, idesc_o, 1u);
                    }
                }
                if (!ok) break;
                sm100::mma_commit(&bars->v_empty[st]);
                sm100::mma_commit(&bars->o_ready);
            }
            if (ok) sm100::mma_commit(&bars->o_done);
        }
    } else {
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const int q = qt * BM + row;
        const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            if (!sm100::mbar_wait(&bars->s_full[j & 1], (uint32_t)(j >> 1) & 1u, status, 47)) {
                ok = false;
                break;
            }
            sm100::tc_fence_after();
            const int key0 = j * BN;
            const bool masked = (CAUSAL && j == qt) || key0 + BN > S;
            const int lim = masked ? min(CAUSAL && j == qt ? row : BN - 1, S - 1 - key0) : BN - 1;
            const uint32_t sb = tmem + 128u * (uint32_t)(j & 1);
            if (masked)
                softmax_tile_kh<T, D, true>(sb, tmem_o, lane_off, lim, j, scale_log2, m, l, &bars->p_full[j & 1][0], &bars->o_ready, status);
            else
                softmax_tile_kh<T, D, false>(sb, tmem_o, lane_off, lim, j, scale_log2, m, l, &bars->p_full[j & 1][0], &bars->o_ready, status);
        }
        if (ok && nkv > 0 && sm100::mbar_wait(&bars->o_done, 0, status, 49)) {
            sm100::tc_fence_after();
            const float inv = 1.0f / l;
            T* orow = o + ((int64_t)bh * S + q) * D;
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem_o + lane_off + (uint32_t)(c * 32), r);
                sm100::tmem_ld_wait();
                if (q < S) {
                    uint4* d4 = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        d4[i] = make_uint4(pack2<T>(__uint_as_float(r[8 * i + 0]) * inv, __uint_as_float(r[8 * i + 1]) * inv),
                                           pack2<T>(__uint_as_float(r[8 * i + 2]) * inv, __uint_as_float(r[8 * i + 3]) * inv),
                                           pack2<T>(__uint_as_float(r[8 * i + 4]) * inv, __uint_as_float(r[8 * i + 5]) * inv),
                                           pack2<T>(__uint_as_float(r[8 * i + 6]) * inv, __uint_as_float(r[8 * i + 7]) * inv));
                }
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 1) sm100::tmem_dealloc(tmem, DB_TMEM_COLS);
}

// ---- general fallback: one warp per query row, fp32, any D <= 256 / alignment ------------------
template <typename T>
__global__ void __launch_bounds__(128) fa_fallback_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                                                          T* __restrict__ o, int64_t BH, int64_t S, int64_t D, float scale, bool causal) {
    const int64_t rowid = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (rowid >= BH * S) return;
    const int64_t bh = rowid / S, i = rowid % S;
    const T* qr = q + rowid * D;
    const T* kb = k + bh * S * D;
    const T* vb = v + bh * S * D;
    float acc[8];  // D <= 256: lane owns d = lane + 32*t
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = 0.f;
    float m = -INFINITY, l = 0.f;
    const int64_t jend = causal ? i + 1 : S;
    for (int64_t j = 0; j < jend; ++j) {
        float part = 0.f;
        for (int64_t d = lane; d < D; d += 32) part += sf::Dt<T>::to_f(qr[d]) * sf::Dt<T>::to_f(kb[j * D + d]);
        const float sc = sf::warp_sum(part) * scale;
        const float m_new = nan_max(m, sc);
        const float a = exp2f((m - m_new) * 1.4426950408889634f);
        const float p = exp2f((sc - m_new) * 1.4426950408889634f);
        l = l * a + p;
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const int64_t d = lane + 32 * t;
            const float vv = d < D ? sf::Dt<T>::to_f(vb[j * D + d]) : 0.f;
            acc[t] = acc[t] * a + p * vv;
        }
        m = m_new;
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const int64_t d = lane + 32 * t;
        if (d < D) o[rowid * D + d] = sf::Dt<T>::from_f(acc[t] / l);
    }
}

sm100::KernelStatus* status_ptr() {
    sm100::KernelStatus* p = nullptr;
    if (cudaGetSymbolAddress((void**)&p, g_attn_status) != cudaSuccess) return nullptr;
    return p;
}

int tmap_bhsd(CUtensorMap* out, const void* base, int64_t BH, int64_t S, int64_t D, bool bf16, char* err, uint64_t cap);

template <typename T, int D, bool CAUSAL>
int launch_db_t(const void* q, const void* k, const void* v, void* o, int64_t BH, int64_t S, float scale, cudaStream_t st, char* err,
                uint64_t cap) {
    const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    CUtensorMap mq, mk, mv;
    int rc = tmap_bhsd(&mq, q, BH, S, D, bf16, err, cap);
    if (!rc) rc = tmap_bhsd(&mk, k, BH, S, D, bf16, err, cap);
    if (!rc) rc = tmap_bhsd(&mv, v, BH, S, D, bf16, err, cap);
    if (rc) return rc;
    sm100::KernelStatus* status = status_ptr();
    if (!status) return sf::fail(SF_EDEVICE, err, cap, "attention: cannot resolve the status word");
    // One CTA per SM: all 512 TMEM columns, and more than half the shared memory so that a second
    // CTA (which would wait for TMEM) is never co-resident.
    const int smem = std::max(LayoutDB<D>::BYTES + 1024, 120 * 1024);
    static std::atomic<uint64_t> attr_done{0};
    if (sf::once_per_device(attr_done))
        cudaFuncSetAttribute(fa_fwd_db_kernel<T, D, CAUSAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    const int64_t nq = (S + BM - 1) / BM;
    if (BH > 0x7fffffffLL || nq > 0x7fffffffLL || BH * nq > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "attention: grid too large");
    const int64_t kv_head = 4 * S * D;
    const int group = (int)std::max<int64_t>(1, std::min<int64_t>({16, BH, (32LL << 20) / std::max<int64_t>(kv_head, 1)}));
    fa_fwd_db_kernel<T, D, CAUSAL><<<(unsigned)(BH * nq), NUM_THREADS, smem, st>>>(mq, mk, mv, (T*)o, (int)S, (int)BH, (int)nq, group,
                                                                                  scale * 1.4426950408889634f, status);
    return sf::check_launch("attention launch", err, cap);
}

template <typename T, int D, bool CAUSAL>
int launch_tc_t(const void* q, const void* k, const void* v, void* o, int64_t BH, int64_t S, float scale, cudaStream_t st, char* err,
                uint64_t cap) {
    const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    CUtensorMap mq, mk, mv;
    int rc = tmap_bhsd(&mq, q, BH, S, D, bf16, err, cap);
    if (!rc) rc = tmap_bhsd(&mk, k, BH, S, D, bf16, err, cap);
    if (!rc) rc = tmap_bhsd(&mv, v, BH, S, D, bf16, err, cap);
    if (rc) return rc;
    sm100::KernelStatus* status = status_ptr();
    if (!status) return sf::fail(SF_EDEVICE, err, cap, "attention: cannot resolve the status word");
    // Two CTAs per SM: 2 x 256 TMEM columns, and at least 80 KB of shared memory each so that a
    // third CTA (which would wait for TMEM) is never co-resident.
    const int smem = std::max(Layout<D>::BYTES + 1024, 80 * 1024);
    static std::atomic<uint64_t> attr_done{0};
    if (sf::once_per_device(attr_done))
        cudaFuncSetAttribute(fa_fwd_kernel<T, D, CAUSAL>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    const int64_t nq = (S + BM - 1) / BM;
    if (BH > 0x7fffffffLL || nq > 0x7fffffffLL || BH * nq > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "attention: grid too large");
    // Heads per group: K and V of a group (2 * S * D * 2 bytes per head) stay within ~32 MB of L2.
    const int64_t kv_head = 4 * S * D;
    const int group = (int)std::max<int64_t>(1, std::min<int64_t>({16, BH, (32LL << 20) / std::max<int64_t>(kv_head, 1)}));
    fa_fwd_kernel<T, D, CAUSAL><<<(unsigned)(BH * nq), NUM_THREADS, smem, st>>>(mq, mk, mv, (T*)o, (int)S, (int)BH, (int)nq, group,
                                                                               scale * 1.4426950408889634f, status);
    return sf::check_launch("attention launch", err, cap);
}

template <typename T>
int launch_t(const void* q, const void* k, const void* v, void* o, int64_t BH, int64_t S, int64_t D, float scale, bool causal,
             int32_t variant, cudaStream_t st, char* err, uint64_t cap) {
    const bool tc = (D == 64 || D == 128) && sf::aligned16(q) && sf::aligned16(k) && sf::aligned16(v) && sf::aligned16(o) &&
                    S < (1LL << 31) && BH < (1LL << 31);
    if ((variant == 1 || variant == 3) && !tc) return sf::fail(SF_EINVAL, err, cap, "attention: the tensor-core variant needs D in {64,128} and aligned tensors");
    // Variant 3, or by default a grid of at most one (b*h, query tile) CTA per SM: the kernel that
    // overlaps Q.K with the softmax inside the CTA.
    const int64_t ctas = BH * ((S + BM - 1) / BM);
    if (tc && (variant == 3 || (variant == 0 && ctas <= (int64_t)sf::sm_count()))) {
        if (D == 64)
            return causal ? launch_db_t<T, 64, true>(q, k, v, o, BH, S, scale, st, err, cap)
                          : launch_db_t<T, 64, false>(q, k, v, o, BH, S, scale, st, err, cap);
        return causal ? launch_db_t<T, 128, true>(q, k, v, o, BH, S, scale, st, err, cap)
                      : launch_db_t<T, 128, false>(q, k, v, o, BH, S, scale, st, err, cap);
    }
    if (tc && variant != 2) {
        if (D == 64)
            return causal ? launch_tc_t<T, 64, true>(q, k, v, o, BH, S, scale, st, err, cap)
                          : launch_tc_t<T, 64, false>(q, k, v, o, BH, S, scale, st, err, cap);
        return causal ? launch_tc_t<T, 128, true>(q, k, v, o, BH, S, scale, st, err, cap)
                      : launch_tc_t<T, 128, false>(q, k, v, o, BH, S, scale, st, err, cap);
    }
    if (D > 256) return sf::fail(SF_EINVAL, err, cap, "attention: D=%lld exceeds the general kernel's 256", (long long)D);
    const int64_t rows = BH * S;
    fa_fallback_kernel<T><<<(unsigned)((rows + 3) / 4), 128, 0, st>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, BH, S, D, scale, causal);
    return sf::check_launch("attention fallback launch", err, cap);
}

int tmap_bhsd(CUtensorMap* out, const void* base, int64_t BH, int64_t S, int64_t D, bool bf16, char* err, uint64_t cap) {
    return sf::tmap_3d(out, base, D, S, BH, D * 2, S * D * 2, 64, BM, 1, bf16, err, cap);
}

}  // namespace

int sf_attention_launch(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H, int64_t S, int64_t D, float scale,
                        int32_t causal, int32_t dtype, int32_t variant, cudaStream_t st, char* err, uint64_t cap) {
    if (B < 0 || H < 0 || S < 0 || D < 1) return sf::fail(SF_EINVAL, err, cap, "attention: bad sizes");
    if (!(scale > 0.f)) return sf::fail(SF_EINVAL, err, cap, "attention: scale must be > 0");
    if (B * H * S == 0) return SF_OK;
    if (!q || !k || !v || !o) return sf::fail(SF_EINVAL, err, cap, "attention: null tensor pointer");
    if (dtype == SF_DTYPE_F16) return launch_t<__half>(q, k, v, o, B * H, S, D, scale, causal != 0, variant, st, err, cap);
    if (dtype == SF_DTYPE_BF16) return launch_t<__nv_bfloat16>(q, k, v, o, B * H, S, D, scale, causal != 0, variant, st, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "attention: dtype %d is not fp16/bf16", dtype);
}

int sf_attention_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream) {
    sm100::KernelStatus h{0, 0};
    if (cudaMemcpyFromSymbolAsync(&h, g_attn_status, sizeof(h), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess) return SF_EDEVICE;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return SF_EDEVICE;
    if (h.code) {
        const sm100::KernelStatus zero{0, 0};
        cudaMemcpyToSymbolAsync(g_attn_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream);
        cudaStreamSynchronize(stream);
    }
    *code = h.code;
    *where = h.where;
    return SF_OK;
}

extern "C" int sf_flash_attention(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H, int64_t S, int64_t D,
                                  float scale, int32_t causal, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_attention_launch(q, k, v, o, B, H, S, D, scale, causal, dtype, 0, (cudaStream_t)stream, err, cap);
}
