// BitDelta GEMMs on the tcgen05 tensor cores, sm_100a.  The +-1 sign operand is never stored
// in HBM: its packed bits are expanded straight into a 128-byte-swizzled K-major shared-memory
// tile that tcgen05.mma reads like any TMA-loaded operand.
//
// Task contract (tasks/bitdelta_gemm/reference.py:99-130, opspec.json:5):
//   y[M,N] = SCALE * x[M,K] . W[K,N],  W[k,n] = +1 if bit (k % 32) of bits[k/32, n] is set, else -1
//   -> bitdelta_task_kernel: 128x128 output tiles, A = x (TMA), B = signs expanded from the
//      [KB, N] words of each K-block, fp32 accumulation in TMEM, SCALE in the epilogue.
//
// W_base variant (the 1-bit-delta fine-tune workload):
//   y[M,N] = x[M,K] . (W_base[N,K] + diag(alpha[N]) S[N,K])^T = x.W_base^T + alpha (x) (x.S^T)
//   S in {-1,+1} packed along K: bit j of S_words[n, kb] is S[n, kb*32 + j].
//   -> bitdelta_base_kernel: M <= 128 rows make the op HBM-bound (W_base is 2*N*K bytes read
//      once), so the product is computed transposed (swap-AB): each CTA owns 128 output columns
//      n, A = W_base rows (TMA) and A' = S rows (expanded), B = x (TMA, M padded to a multiple of
//      16 with zero rows), two TMEM accumulators D1 = W_base.x^T and D2 = S.x^T (the +-1 products
//      are exact in fp32), epilogue p = D1 + alpha[n] * D2.  K is split over the CTAs of a
//      thread-block cluster (up to 8) so ~all SMs stream W_base; the partials are reduce-scattered
//      through distributed shared memory (each CTA sums a slice of the M rows of y from every
//      peer's partial and writes it).  No workspace.
//
// One to four rows of x take a streaming kernel instead (bitdelta_base_stream_kernel, below): a
// matrix-vector stream over W_base and the sign words, no tensor cores.
//
// Sign expansion uses a 256-entry shared-memory table: one 16-byte lookup per 8 signs.  The
// base kernel keeps 8 interleaved copies of the table (entry e of copy k at 16-byte slot
// 8e + k) and lane L reads copy L % 8, so the 8 lanes of each 128-bit shared-memory phase hit 8
// different bank groups whatever bytes they look up.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + MMA issuer, warps 2..5
// expand sign bits for every stage and run the epilogue.  Every mbarrier wait is bounded.
// The base kernel streams W_base (+ x) through a deep TMA ring (up to 8 stages) and the expanded
// signs through a separate 3-entry ring, so DRAM sees up to 8 W_base tiles in flight per SM.
#include "sf_common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <cudaTypedefs.h>
#include <algorithm>
#include <mutex>
#include <type_traits>

__device__ sm100::KernelStatus g_bitdelta_status;

namespace {

constexpr int BK = 64;
constexpr int TILE_ROWS = 128;
constexpr int ROW_TILE_BYTES = TILE_ROWS * BK * 2;  // 16 KB: 128 rows x 128 bytes
constexpr int NUM_THREADS = 192;
// The base kernel adds a seventh warp: warp 1 issues the W_base MMAs and warp 6 the sign MMAs,
// into their separate accumulators (one thread's tcgen05.mma issue is the per-K-block limit).
constexpr int BASE_THREADS = 224;
constexpr int SMEM_LIMIT = 227 * 1024;
// Neither kernel has static shared memory (the sign tables are dynamic).
constexpr int BASE_SMEM_LIMIT = SMEM_LIMIT;

constexpr int TASK_MAX_STAGES = 8;

struct __align__(8) Bars {
    uint64_t full_tma[TASK_MAX_STAGES];
    uint64_t full_exp[TASK_MAX_STAGES];
    uint64_t empty[TASK_MAX_STAGES];
    uint64_t acc_full;
    uint32_t tmem_base;
};
static_assert(sizeof(Bars) <= 256, "the task kernel reserves 256 bytes for its barriers");

constexpr int BASE_MAX_STAGES = 8;  // W_base + x ring
constexpr int BASE_SSTAGES = 3;     // expanded-sign ring
constexpr int LUT_COPIES = 8;
constexpr int LUT8_BYTES = 256 * LUT_COPIES * 16;

struct __align__(8) BaseBars {
    uint64_t full_w[BASE_MAX_STAGES];
    uint64_t empty_w[BASE_MAX_STAGES];
    uint64_t full_s[BASE_SSTAGES];
    uint64_t empty_s[BASE_SSTAGES];
    uint64_t acc_full;
    uint32_t tmem_base;
};

template <typename T>
__device__ __forceinline__ uint32_t minus_one_pair() {
    return std::is_same<T, __half>::value ? 0xBC00BC00u : 0xBF80BF80u;
}

// Lookup table: byte value b -> the 8 16-bit values (+1 where bit j of b is set, else -1) of one
// 16-byte chunk, built once per CTA in shared memory as LUT_COPIES interleaved copies: slot 8e + k
// holds entry e.
template <typename T>
__device__ __forceinline__ void build_sign_lut8(uint4* lut) {
    const uint32_t base = minus_one_pair<T>();
    for (int i = threadIdx.x; i < 256 * LUT_COPIES; i += blockDim.x) {
        const uint32_t e = (uint32_t)i / LUT_COPIES;
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t b = (e >> (2 * q)) & 3u;
            w[q] = base ^ ((b & 1u) << 15) ^ ((b & 2u) << 30);
        }
        lut[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Row r of a K-major 128-byte-swizzled tile (64 16-bit elements per row) from 64 sign bits, reading
// copy `copy` of the interleaved table: element j = +1 if bit j is set, else -1; chunk c (elements
// 8c..8c+7) lives at chunk c ^ (r % 8).
__device__ __forceinline__ void expand_row_sw128_lut8(uint8_t* tile, int r, uint64_t bits, const uint4* lut, int copy) {
    uint8_t* row = tile + r * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) * 16)) = lut[(((uint32_t)(bits >> (8 * c)) & 0xFFu) << 3) + copy];
    }
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

// ------------------------------------------------------------------------------------------------
// W_base variant (swap-AB, split-K over a cluster)
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(BASE_THREADS, 1)
    bitdelta_base_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                         const uint32_t* __restrict__ s_words, const T* __restrict__ alpha, T* __restrict__ y, int M, int N,
                         int K, int nm, int stages, int vec_words, int tile_n, sm100::KernelStatus* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int x_bytes = nm * 128;
    const int w_bytes = tile_n * 128;                         // rows of W_base this CTA owns
    const int stage_bytes = ROW_TILE_BYTES + x_bytes;        // W_base tile + x tile
    uint8_t* sring = smem + stages * stage_bytes;             // expanded signs
    uint4* lut = reinterpret_cast<uint4*>(sring + BASE_SSTAGES * ROW_TILE_BYTES);
    BaseBars* bars = reinterpret_cast<BaseBars*>(reinterpret_cast<uint8_t*>(lut) + LUT8_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * tile_n;
    const int sk = gridDim.y;
    const uint32_t rank = sm100::cluster_ctarank();
    const int nkb = (K + BK - 1) / BK;
    const int kb_begin = (int)((int64_t)nkb * rank / sk);
    const int kb_end = (int)((int64_t)nkb * (rank + 1) / sk);
    const int kw = K / 32;  // words per S row
    const uint32_t tmem_cols = (uint32_t)max(32, 1 << (32 - __clz(2 * nm - 1)));

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            sm100::mbar_init(&bars->full_w[s], 1);
            sm100::mbar_init(&bars->empty_w[s], 2);  // both MMA issuers read the stage's x tile
        }
        for (int s = 0; s < BASE_SSTAGES; ++s) {
            sm100::mbar_init(&bars->full_s[s], 128);
            sm100::mbar_init(&bars->empty_s[s], 1);
        }
        sm100::mbar_init(&bars->acc_full, 2);
        sm100::fence_mbar_init();
    }
    // Sign words of the first 16 K-blocks are requested first, then (after a CTA barrier, so the
    // memory system sees them ahead of every CTA's burst of W_base tiles) the first ring of W_base /
    // x tiles; both latencies overlap the table build and TMEM allocation.
    const int pre = min(stages, max(kb_end - kb_begin, 0));
    auto issue = [&](int kb, int s) {
        uint8_t* st = smem + s * stage_bytes;
        sm100::mbar_arrive_expect_tx(&bars->full_w[s], w_bytes + x_bytes);
        sm100::tma_load_2d(st, &tmap_w, &bars->full_w[s], kb * BK, n0);
        sm100::tma_load_2d(st + ROW_TILE_BYTES, &tmap_x, &bars->full_w[s], kb * BK, 0);
    };
    const bool expander = warp >= 2 && warp < 6;  // warps 2..5: sign expansion and the epilogue
    const int t = threadIdx.x - 64;
    const int n = n0 + t;
    const bool row_live = expander && t < tile_n && n < N;
    uint32_t wv[32];
    auto load_words = [&](int kc) {
        const int w0 = 2 * kc;
        const uint32_t* src = s_words + (int64_t)n * kw + w0;
        if (vec_words && row_live && kc + 16 <= kb_end && (w0 & 3) == 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + i);
                wv[4 * i] = v.x;
                wv[4 * i + 1] = v.y;
                wv[4 * i + 2] = v.z;
                wv[4 * i + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) wv[i] = (row_live && w0 + i < 2 * kb_end && w0 + i < kw) ? __ldg(src + i) : 0u;
        }
    };
    if (expander && kb_end > kb_begin) load_words(kb_begin);
    __syncthreads();  // barrier initialisation visible; the sign-word loads issued
    if (threadIdx.x == 0) {
        sm100::tma_prefetch_desc(&tmap_w);
        sm100::tma_prefetch_desc(&tmap_x);
        for (int i = 0; i < pre; ++i) issue(kb_begin + i, i);
    }
    build_sign_lut8<T>(lut);
    if (warp == 1) {
        sm100::tmem_alloc(&bars->tmem_base, tmem_cols);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            int s = pre % stages;
            uint32_t ph = pre == stages ? 1u : 0u;
            for (int kb = kb_begin + pre; kb < kb_end; ++kb) {
                if (!sm100::mbar_wait(&bars->empty_w[s], ph ^ 1u, status, 11)) break;
                issue(kb, s);
                if (++s == stages) { s = 0; ph ^= 1u; }
            }
        }
    } else if (warp == 1 || warp == 6) {
        // Warp 1: D1 = W_base . x^T; warp 6: D2 = S . x^T (waits for the expanded S tile too).
        // Each releases the W_base / x stage (two arrivals) and warp 6 the S stage.
        if (lane == 0 && kb_end > kb_begin) {
            const bool sign = warp == 6;
            const uint32_t idesc = sm100::idesc_f16(128, (uint32_t)nm, std::is_same<T, __nv_bfloat16>::value);
            const uint32_t dst = tmem + (sign ? (uint32_t)nm : 0u);
            int s = 0, e = 0;
            uint32_t ph = 0, phe = 0;
            bool ok = true;
            for (int kb = kb_begin; kb < kb_end; ++kb) {
                if (!sm100::mbar_wait(&bars->full_w[s], ph, status, 12) ||
                    (sign && !sm100::mbar_wait(&bars->full_s[e], phe, status, 13))) {
                    ok = false;
                    break;
                }
                sm100::tc_fence_after();
                const uint32_t sw = sm100::smem_u32(smem + s * stage_bytes);
                const uint32_t sx = sw + ROW_TILE_BYTES;
                const uint32_t sa = sign ? sm100::smem_u32(sring + e * ROW_TILE_BYTES) : sw;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)
                    sm100::mma_f16(dst, sm100::smem_desc_k_sw128(sa + k * 32), sm100::smem_desc_k_sw128(sx + k * 32), idesc,
                                   (kb > kb_begin || k > 0) ? 1u : 0u);
                sm100::mma_commit(&bars->empty_w[s]);
                if (sign) sm100::mma_commit(&bars->empty_s[e]);
                if (++s == stages) { s = 0; ph ^= 1u; }
                if (++e == BASE_SSTAGES) { e = 0; phe ^= 1u; }
            }
            if (ok) sm100::mma_commit(&bars->acc_full);
        }
    } else {
        // Sign expansion: thread t owns row t (output column n0 + t) of every S tile.  The sign
        // words of 16 K-blocks are loaded up front (independent loads, one memory latency per 16
        // stages instead of one per stage), as 16-byte vectors when the rows allow it.  Rows at
        // or past tile_n are not this CTA's: their S rows are left as they are (the MMA rows
        // they feed are never read).
        const int copy = lane & (LUT_COPIES - 1);
        int e = 0;
        uint32_t phe = 0;
        bool ok = true;
        for (int kc = kb_begin; kc < kb_end && ok; kc += 16) {
            if (kc != kb_begin) load_words(kc);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (kc + i >= kb_end) break;
                if (!sm100::mbar_wait(&bars->empty_s[e], phe ^ 1u, status, 14)) {
                    ok = false;
                    break;
                }
                if (t < tile_n)
                    expand_row_sw128_lut8(sring + e * ROW_TILE_BYTES, t, (uint64_t)wv[2 * i] | ((uint64_t)wv[2 * i + 1] << 32), lut, copy);
                sm100::fence_proxy_async_smem();
                sm100::mbar_arrive(&bars->full_s[e]);
                if (++e == BASE_SSTAGES) { e = 0; phe ^= 1u; }
            }
        }
    }

    // ---- epilogue: partial p[row][m] = D1 + alpha[n] * D2 into shared memory (the pipeline
    // buffers are free once acc_full has fired: every MMA reading them has completed).
    float* red = reinterpret_cast<float*>(smem);
    if (expander) {
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const int n = n0 + row;
        const float a = (row < tile_n && n < N) ? sf::Dt<T>::to_f(alpha[n]) : 0.f;
        bool have = kb_end > kb_begin;
        if (have && !sm100::mbar_wait(&bars->acc_full, 0, status, 15)) have = false;
        sm100::tc_fence_after();
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        for (int c = 0; c < nm; c += 16) {
            float p[16];
            if (have) {
                uint32_t d1[16], d2[16];
                sm100::tmem_ld_32x32b_x16(lane_base + (uint32_t)c, d1);
                sm100::tmem_ld_32x32b_x16(lane_base + (uint32_t)(nm + c), d2);
                sm100::tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) p[j] = __uint_as_float(d1[j]) + a * __uint_as_float(d2[j]);
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) p[j] = 0.f;
            }
            float4* dst = reinterpret_cast<float4*>(red + (size_t)row * nm + c);
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[j] = make_float4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
        }
    }
    __syncthreads();
    sm100::cluster_sync();  // every CTA's partial is in its shared memory
    // Reduce-scatter over the cluster: CTA `rank` sums the columns [c0, c1) of all partials
    // (16-byte loads through distributed shared memory) and writes those rows of y.
    if (expander) {
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const int n = n0 + row;
        const int per = (((M + sk - 1) / sk) + 3) & ~3;
        const int c0 = (int)rank * per;
        const int c1 = min(M, c0 + per);
        if (row < tile_n && n < N) {
            const uint32_t own = sm100::smem_u32(red + (size_t)row * nm);
            for (int c = c0; c < c1; c += 4) {
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int r = 0; r < sk; ++r) {
                    const float4 v = sm100::ld_shared_cluster_v4(sm100::mapa_shared(own + 4u * c, (uint32_t)r));
                    acc.x += v.x;
                    acc.y += v.y;
                    acc.z += v.z;
                    acc.w += v.w;
                }
                const float o[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (c + j < c1) y[(int64_t)(c + j) * N + n] = sf::Dt<T>::from_f(o[j]);
            }
        }
    }
    sm100::cluster_sync();  // every CTA keeps its shared memory until all peers have read it
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 1) sm100::tmem_dealloc(tmem, tmem_cols);
}

// ------------------------------------------------------------------------------------------------
// Task contract: y = SCALE * x . W, W from bits [KB, N]
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    bitdelta_task_kernel(const __grid_constant__ CUtensorMap tmap_x, const uint32_t* __restrict__ bits, T* __restrict__ y, int M,
                         int N, int K, float scale, int stages, sm100::KernelStatus* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int stage_bytes = 2 * ROW_TILE_BYTES;
    Bars* bars = reinterpret_cast<Bars*>(smem + stages * stage_bytes);
    // Sign table with LUT_COPIES interleaved copies (lane L reads copy L % 8: the 8 lanes of a
    // 128-bit shared-memory phase hit 8 bank groups).
    uint4* lut = reinterpret_cast<uint4*>(smem + stages * stage_bytes + 256);
    build_sign_lut8<T>(lut);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * TILE_ROWS, n0 = blockIdx.x * TILE_ROWS;
    const int nkb = (K + BK - 1) / BK;
    const int kbw = K / 32;  // rows of the bits array
    constexpr uint32_t TMEM_COLS = 128;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            sm100::mbar_init(&bars->full_tma[s], 1);
            sm100::mbar_init(&bars->full_exp[s], 128);
            sm100::mbar_init(&bars->empty[s], 1);
        }
        sm100::mbar_init(&bars->acc_full, 1);
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

    if (warp == 0) {
        if (lane == 0) {
            sm100::tma_prefetch_desc(&tmap_x);
            int s = 0;
            uint32_t ph = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                if (!sm100::mbar_wait(&bars->empty[s], ph ^ 1u, status, 21)) break;
                sm100::mbar_arrive_expect_tx(&bars->full_tma[s], ROW_TILE_BYTES);
                sm100::tma_load_2d(smem + s * stage_bytes, &tmap_x, &bars->full_tma[s], kb * BK, m0);
                if (++s == stages) { s = 0; ph ^= 1u; }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = sm100::idesc_f16(128, 128, std::is_same<T, __nv_bfloat16>::value);
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            for (int kb = 0; kb < nkb; ++kb) {
                if (!sm100::mbar_wait(&bars->full_tma[s], ph, status, 22) || !sm100::mbar_wait(&bars->full_exp[s], ph, status, 23)) {
                    ok = false;
                    break;
                }
                sm100::tc_fence_after();
                const uint32_t sa = sm100::smem_u32(smem + s * stage_bytes);
                const uint32_t sb = sa + ROW_TILE_BYTES;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)
                    sm100::mma_f16(tmem, sm100::smem_desc_k_sw128(sa + k * 32), sm100::smem_desc_k_sw128(sb + k * 32), idesc,
                                   (kb > 0 || k > 0) ? 1u : 0u);
                sm100::mma_commit(&bars->empty[s]);
                if (++s == stages) { s = 0; ph ^= 1u; }
            }
            if (ok) sm100::mma_commit(&bars->acc_full);
        }
    } else {
        const int t = threadIdx.x - 64;
        const int n = n0 + t;
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int kc = 0; kc < nkb && ok; kc += 16) {
            uint32_t lo[16], hi[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int w = 2 * (kc + i);
                const bool live = n < N && kc + i < nkb;
                lo[i] = (live && w < kbw) ? bits[(int64_t)w * N + n] : 0u;
                hi[i] = (live && w + 1 < kbw) ? bits[(int64_t)(w + 1) * N + n] : 0u;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (kc + i >= nkb) break;
                if (!sm100::mbar_wait(&bars->empty[s], ph ^ 1u, status, 24)) {
                    ok = false;
                    break;
                }
                expand_row_sw128_lut8(smem + s * stage_bytes + ROW_TILE_BYTES, t, (uint64_t)lo[i] | ((uint64_t)hi[i] << 32), lut,
                                      lane & (LUT_COPIES - 1));
                sm100::fence_proxy_async_smem();
                sm100::mbar_arrive(&bars->full_exp[s]);
                if (++s == stages) { s = 0; ph ^= 1u; }
            }
        }
        // epilogue: TMEM lane = output row m, columns = n.
        const int quad = warp & 3;
        const int m = m0 + quad * 32 + lane;
        if (sm100::mbar_wait(&bars->acc_full, 0, status, 25)) {
            sm100::tc_fence_after();
            const bool vec_ok = (N % 8) == 0;
            for (int c = 0; c < 128; c += 32) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c, r);
                sm100::tmem_ld_wait();
                const int col0 = n0 + c;
                if (m < M) {
                    T* dst = y + (int64_t)m * N + col0;
                    if (vec_ok && col0 + 32 <= N) {
                        uint32_t p[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            p[j] = pack2<T>(scale * __uint_as_float(r[2 * j]), scale * __uint_as_float(r[2 * j + 1]));
                        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                        for (int j = 0; j < 4; ++j) d4[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
                    } else {
                        for (int j = 0; j < 32; ++j)
                            if (col0 + j < N) dst[j] = sf::Dt<T>::from_f(scale * __uint_as_float(r[j]));
                    }
                }
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 1) sm100::tmem_dealloc(tmem, TMEM_COLS);
}

// ------------------------------------------------------------------------------------------------
// General fallbacks (any shape / alignment): one thread per output element, fp32 accumulation.
// ------------------------------------------------------------------------------------------------
template <typename T>
__global__ void bitdelta_task_fallback(const T* __restrict__ x, const uint32_t* __restrict__ bits, T* __restrict__ y, int64_t M,
                                       int64_t N, int64_t K, float scale) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= M * N) return;
    const int64_t m = idx / N, n = idx % N;
    float acc = 0.f;
    for (int64_t k = 0; k < K; ++k) {
        const uint32_t w = bits[(k >> 5) * N + n];
        const float sgn = ((w >> (k & 31)) & 1u) ? 1.f : -1.f;
        acc = fmaf(sf::Dt<T>::to_f(x[m * K + k]), sgn, acc);
    }
    y[idx] = sf::Dt<T>::from_f(scale * acc);
}

template <typename T>
__global__ void bitdelta_base_fallback(const T* __restrict__ x, const T* __restrict__ wb, const uint32_t* __restrict__ sw,
                                       const T* __restrict__ alpha, T* __restrict__ y, int64_t M, int64_t N, int64_t K) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= M * N) return;
    const int64_t m = idx / N, n = idx % N;
    const int64_t kw = K / 32;
    float a1 = 0.f, a2 = 0.f;
    for (int64_t k = 0; k < K; ++k) {
        const float xv = sf::Dt<T>::to_f(x[m * K + k]);
        a1 = fmaf(xv, sf::Dt<T>::to_f(wb[n * K + k]), a1);
        const uint32_t w = sw[n * kw + (k >> 5)];
        a2 += ((w >> (k & 31)) & 1u) ? xv : -xv;
    }
    y[idx] = sf::Dt<T>::from_f(a1 + sf::Dt<T>::to_f(alpha[n]) * a2);
}

// ---- few-row streaming kernel (M <= 4) -----------------------------------------------------------
// For one to four rows of x the product is a matrix-vector stream over W_base (2NK bytes) and the
// packed signs (NK/8 bytes): one warp per output column n (a row of W_base), lanes streaming
// 16-byte vectors of that row with four in flight before the first multiply-add, the 8 signs of a
// vector taken from one byte of its 32-bit sign word (bit j of S_words[n, k/32] is S[n, k], k = 8v
// + j for vector v), x read through L1 (every warp reads the same x).  fp32 accumulators of
// x.W_base^T and x.S^T per row, a shuffle reduction, y = acc_w + alpha[n] acc_s: the same two
// products and the same combination as the tensor-core kernel.
constexpr int STREAM_WARPS = 4;
constexpr int STREAM_UNROLL = 4;

template <typename T, int MR>
__global__ void __launch_bounds__(STREAM_WARPS * 32, MR == 1 ? 8 : 4)
    bitdelta_base_stream_kernel(const T* __restrict__ x, const T* __restrict__ wb, const uint32_t* __restrict__ sw,
                                const T* __restrict__ alpha, T* __restrict__ y, int64_t N, int64_t K) {
    const int lane = threadIdx.x & 31;
    const int64_t kv = K >> 3, kw = K >> 5;
    const int64_t wstride = (int64_t)gridDim.x * STREAM_WARPS;
    for (int64_t n = (int64_t)blockIdx.x * STREAM_WARPS + (threadIdx.x >> 5); n < N; n += wstride) {
        const T* row = wb + n * K;
        const uint32_t* srow = sw + n * kw;
        float aw[MR], as[MR];
#pragma unroll
        for (int m = 0; m < MR; ++m) aw[m] = as[m] = 0.f;
        for (int64_t v0 = lane; v0 < kv; v0 += 32 * STREAM_UNROLL) {
            sf::Vec8<T> w[STREAM_UNROLL];
            uint32_t bits[STREAM_UNROLL];
#pragma unroll
            for (int u = 0; u < STREAM_UNROLL; ++u) {
                const int64_t v = v0 + 32 * u;
                if (v < kv) {
                    w[u] = sf::ld_global_nc_v8<T>(row + v * 8);
                    bits[u] = __ldg(srow + (v >> 2)) >> (8 * (v & 3));
                }
            }
#pragma unroll
            for (int u = 0; u < STREAM_UNROLL; ++u) {
                const int64_t v = v0 + 32 * u;
                if (v < kv) {
#pragma unroll
                    for (int m = 0; m < MR; ++m) {
                        sf::Vec8<T> xv;
                        *reinterpret_cast<uint4*>(&xv) = __ldg(reinterpret_cast<const uint4*>(x + m * K + v * 8));
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float xf = sf::Dt<T>::to_f(xv.v[j]);
                            aw[m] = fmaf(sf::Dt<T>::to_f(w[u].v[j]), xf, aw[m]);
                            as[m] += ((bits[u] >> j) & 1u) ? xf : -xf;
                        }
                    }
                }
            }
        }
        const float al = sf::Dt<T>::to_f(alpha[n]);
#pragma unroll
        for (int m = 0; m < MR; ++m) {
            float a = aw[m], b = as[m];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                a += __shfl_xor_sync(0xffffffffu, a, off);
                b += __shfl_xor_sync(0xffffffffu, b, off);
            }
            if (lane == 0) y[m * N + n] = sf::Dt<T>::from_f(a + al * b);
        }
    }
}

// ---- host ----------------------------------------------------------------------------------------

sm100::KernelStatus* status_ptr() {
    sm100::KernelStatus* p = nullptr;
    if (cudaGetSymbolAddress((void**)&p, g_bitdelta_status) != cudaSuccess) return nullptr;
    return p;
}

template <typename T>
int launch_base_tc(const void* x, const void* wb, const void* sw, const void* alpha, void* y, int64_t M, int64_t N, int64_t K,
                   cudaStream_t st, char* err, uint64_t cap) {
    const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    sm100::KernelStatus* status = status_ptr();
    if (!status) return sf::fail(SF_EDEVICE, err, cap, "bitdelta: cannot resolve the status word");
    const int64_t nkb = (K + BK - 1) / BK;
    // Tiling: 128 rows of W_base per CTA (the MMA instruction count per CTA depends only on its
    // share of K, so tiles are kept as tall as the MMA allows) and K split over a cluster of sk
    // CTAs, as many as still fit in one wave (clusters are placed within GPCs, so 4 x 32 = 128
    // CTAs fit on 148 SMs where 4 x 37 do not).
    int tile_n = (int)std::min<int64_t>(TILE_ROWS, std::max<int64_t>(16, (N + 7) / 8 * 8));
    const int64_t ntiles = (N + tile_n - 1) / tile_n;
    int sk = (int)std::max<int64_t>(1, std::min<int64_t>(8, sf::sm_count() / std::max<int64_t>(ntiles, 1)));
    sk = (int)std::min<int64_t>(sk, nkb);
    const int64_t tiles = (N + tile_n - 1) / tile_n;
    CUtensorMap mw;
    int rc = sf::tmap_kmajor(&mw, wb, N, K, tile_n, bf16, err, cap);
    if (rc) return rc;
    // 16-byte sign-word loads when every S row starts on a 16-byte boundary.
    const int vec_words = ((K / 32) % 4 == 0 && sf::aligned16(sw)) ? 1 : 0;
    // x rows are processed in chunks of at most 256 (the MMA N dimension).
    for (int64_t mc = 0; mc < M; mc += 256) {
        const int64_t mrows = std::min<int64_t>(256, M - mc);
        const int nm = (int)((mrows + 15) / 16 * 16);
        CUtensorMap mx;
        rc = sf::tmap_kmajor(&mx, (const T*)x + mc * K, mrows, K, nm, bf16, err, cap);
        if (rc) return rc;
        const int stage_bytes = ROW_TILE_BYTES + nm * 128;
        const int fixed = BASE_SSTAGES * ROW_TILE_BYTES + LUT8_BYTES + (int)sizeof(BaseBars) + 1024;
        const int stages = std::min(BASE_MAX_STAGES, (BASE_SMEM_LIMIT - fixed) / stage_bytes);
        const int smem = stages * stage_bytes + fixed;
        // The reduction buffer (128 x nm fp32) reuses the W_base/x ring and the sign ring.
        if (stages < 2 || 128 * nm * 4 > stages * stage_bytes + BASE_SSTAGES * ROW_TILE_BYTES)
            return sf::fail(SF_EINVAL, err, cap, "bitdelta: no shared-memory plan for M chunk %d", nm);
        static std::atomic<uint64_t> attr_done{0};
        if (sf::once_per_device(attr_done))
            cudaFuncSetAttribute(bitdelta_base_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, BASE_SMEM_LIMIT);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)tiles, (unsigned)sk, 1);
        cfg.blockDim = dim3(BASE_THREADS, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = (unsigned)sk;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e = cudaLaunchKernelEx(&cfg, bitdelta_base_kernel<T>, mw, mx, (const uint32_t*)sw, (const T*)alpha,
                                           (T*)y + mc * N, (int)mrows, (int)N, (int)K, nm, stages, vec_words, tile_n, status);
        if (e != cudaSuccess) return sf::fail(SF_EDEVICE, err, cap, "bitdelta_base launch: %s", cudaGetErrorString(e));
    }
    return SF_OK;
}

template <typename T>
int launch_task_tc(const void* x, const void* bits, void* y, int64_t M, int64_t N, int64_t K, float scale, cudaStream_t st,
                   char* err, uint64_t cap) {
    const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    sm100::KernelStatus* status = status_ptr();
    if (!status) return sf::fail(SF_EDEVICE, err, cap, "bitdelta: cannot resolve the status word");
    CUtensorMap mx;
    int rc = sf::tmap_kmajor(&mx, x, M, K, TILE_ROWS, bf16, err, cap);
    if (rc) return rc;
    const int stages = 5;
    static_assert(5 <= TASK_MAX_STAGES, "one barrier of each kind per stage");
    const int smem = stages * 2 * ROW_TILE_BYTES + 256 + LUT8_BYTES + 1024;
    static std::atomic<uint64_t> attr_done{0};
    if (sf::once_per_device(attr_done))
        cudaFuncSetAttribute(bitdelta_task_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_LIMIT);
    const dim3 grid((unsigned)((N + TILE_ROWS - 1) / TILE_ROWS), (unsigned)((M + TILE_ROWS - 1) / TILE_ROWS));
    if (grid.y > 65535) return sf::fail(SF_EINVAL, err, cap, "bitdelta: M too large");
    bitdelta_task_kernel<T><<<grid, NUM_THREADS, smem, st>>>(mx, (const uint32_t*)bits, (T*)y, (int)M, (int)N, (int)K, scale, stages,
                                                             status);
    return sf::check_launch("bitdelta_task launch", err, cap);
}

bool tc_ok(const void* x, int64_t M, int64_t N, int64_t K) {
    return sf::aligned16(x) && K % 32 == 0 && K > 0 && M > 0 && N > 0 && K < (1LL << 31) && N < (1LL << 31) && M < (1LL << 31);
}

}  // namespace

int sf_bitdelta_base_launch(const void* x, const void* w_base, const void* s_words, const void* alpha, void* y, int64_t M, int64_t N,
                            int64_t K, int32_t dtype, int32_t variant, cudaStream_t st, char* err, uint64_t cap) {
    if (M < 0 || N < 0 || K < 0 || K % 32) return sf::fail(SF_EINVAL, err, cap, "bitdelta_base: need M,N >= 0 and K a multiple of 32");
    if (dtype != SF_DTYPE_F16 && dtype != SF_DTYPE_BF16) return sf::fail(SF_EINVAL, err, cap, "bitdelta_base: dtype %d is not fp16/bf16", dtype);
    if (M == 0 || N == 0) return SF_OK;
    if (!x || !w_base || !s_words || !alpha || !y) return sf::fail(SF_EINVAL, err, cap, "bitdelta_base: null tensor pointer");
    const bool tc = tc_ok(x, M, N, K) && sf::aligned16(w_base);
    // Variant 0: the streaming kernel for M <= 4 (aligned bases), else the tensor-core kernel, else
    // the general kernel; 1 forces the tensor-core kernel, 2 the general one, 3 the streaming one.
    const bool stream = M <= 4 && sf::aligned16(x) && sf::aligned16(w_base) && K > 0;
    if (variant == 3 && !stream) return sf::fail(SF_EINVAL, err, cap, "bitdelta_base: the streaming variant needs M <= 4 and aligned bases");
    if (stream && (variant == 0 || variant == 3)) {
        int64_t blocks = (N + STREAM_WARPS - 1) / STREAM_WARPS;
        const int64_t cap_blocks = (int64_t)sf::sm_count() * (M == 1 ? 8 : 4);
        if (blocks > cap_blocks) blocks = cap_blocks;
#define SF_BITDELTA_STREAM(TT, MRV)                                                                                             \
    bitdelta_base_stream_kernel<TT, MRV><<<(unsigned)blocks, STREAM_WARPS * 32, 0, st>>>((const TT*)x, (const TT*)w_base,        \
                                                                                         (const uint32_t*)s_words,             \
                                                                                         (const TT*)alpha, (TT*)y, N, K)
        if (dtype == SF_DTYPE_F16) {
            switch (M) {
                case 1: SF_BITDELTA_STREAM(__half, 1); break;
                case 2: SF_BITDELTA_STREAM(__half, 2); break;
                case 3: SF_BITDELTA_STREAM(__half, 3); break;
                default: SF_BITDELTA_STREAM(__half, 4); break;
            }
        } else {
            switch (M) {
                case 1: SF_BITDELTA_STREAM(__nv_bfloat16, 1); break;
                case 2: SF_BITDELTA_STREAM(__nv_bfloat16, 2); break;
                case 3: SF_BITDELTA_STREAM(__nv_bfloat16, 3); break;
                default: SF_BITDELTA_STREAM(__nv_bfloat16, 4); break;
            }
        }
#undef SF_BITDELTA_STREAM
        return sf::check_launch("bitdelta_base stream launch", err, cap);
    }
    if (variant == 1 && !tc) return sf::fail(SF_EINVAL, err, cap, "bitdelta_base: the tensor-core variant needs aligned bases");
    if (tc && variant != 2) {
        return dtype == SF_DTYPE_F16 ? launch_base_tc<__half>(x, w_base, s_words, alpha, y, M, N, K, st, err, cap)
                                     : launch_base_tc<__nv_bfloat16>(x, w_base, s_words, alpha, y, M, N, K, st, err, cap);
    }
    const int64_t total = M * N;
    const unsigned blocks = (unsigned)((total + 255) / 256);
    if (dtype == SF_DTYPE_F16)
        bitdelta_base_fallback<__half><<<blocks, 256, 0, st>>>((const __half*)x, (const __half*)w_base, (const uint32_t*)s_words,
                                                               (const __half*)alpha, (__half*)y, M, N, K);
    else
        bitdelta_base_fallback<__nv_bfloat16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)x, (const __nv_bfloat16*)w_base,
                                                                      (const uint32_t*)s_words, (const __nv_bfloat16*)alpha,
                                                                      (__nv_bfloat16*)y, M, N, K);
    return sf::check_launch("bitdelta_base fallback launch", err, cap);
}

int sf_bitdelta_launch(const void* x, const void* bits, void* y, int64_t M, int64_t N, int64_t K, float scale, int32_t dtype,
                       int32_t variant, cudaStream_t st, char* err, uint64_t cap) {
    if (M < 0 || N < 0 || K < 0 || K % 32) return sf::fail(SF_EINVAL, err, cap, "bitdelta: need M,N >= 0 and K a multiple of 32");
    if (dtype != SF_DTYPE_F16 && dtype != SF_DTYPE_BF16) return sf::fail(SF_EINVAL, err, cap, "bitdelta: dtype %d is not fp16/bf16", dtype);
    if (M == 0 || N == 0) return SF_OK;
    if (!x || !bits || !y) return sf::fail(SF_EINVAL, err, cap, "bitdelta: null tensor pointer");
    const bool tc = tc_ok(x, M, N, K);
    if (variant == 1 && !tc) return sf::fail(SF_EINVAL, err, cap, "bitdelta: the tensor-core variant needs an aligned x and K %% 32 == 0");
    if (tc && variant != 2) {
        return dtype == SF_DTYPE_F16 ? launch_task_tc<__half>(x, bits, y, M, N, K, scale, st, err, cap)
                                     : launch_task_tc<__nv_bfloat16>(x, bits, y, M, N, K, scale, st, err, cap);
    }
    const int64_t total = M * N;
    const unsigned blocks = (unsigned)((total + 255) / 256);
    if (dtype == SF_DTYPE_F16)
        bitdelta_task_fallback<__half><<<blocks, 256, 0, st>>>((const __half*)x, (const uint32_t*)bits, (__half*)y, M, N, K, scale);
    else
        bitdelta_task_fallback<__nv_bfloat16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)x, (const uint32_t*)bits,
                                                                      (__nv_bfloat16*)y, M, N, K, scale);
    return sf::check_launch("bitdelta fallback launch", err, cap);
}

int sf_bitdelta_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream) {
    sm100::KernelStatus h{0, 0};
    if (cudaMemcpyFromSymbolAsync(&h, g_bitdelta_status, sizeof(h), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
        return SF_EDEVICE;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return SF_EDEVICE;
    if (h.code) {
        const sm100::KernelStatus zero{0, 0};
        cudaMemcpyToSymbolAsync(g_bitdelta_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream);
        cudaStreamSynchronize(stream);
    }
    *code = h.code;
    *where = h.where;
    return SF_OK;
}

extern "C" int sf_bitdelta_gemm(const void* x, const void* bits, void* y, int64_t M, int64_t N, int64_t K, float scale, int32_t dtype,
                                void* stream, char* err, uint64_t cap) {
    return sf_bitdelta_launch(x, bits, y, M, N, K, scale, dtype, 0, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_bitdelta_gemm_base(const void* x, const void* w_base, const void* s_words, const void* alpha, void* y, int64_t M,
                                     int64_t N, int64_t K, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_bitdelta_base_launch(x, w_base, s_words, alpha, y, M, N, K, dtype, 0, (cudaStream_t)stream, err, cap);
}
