// Mamba-2 SSD chunk scan (one B/C group) on the tcgen05 tensor cores, sm_100a.
//
//   y[b,t,h,:] = sum_{s <= t, s in chunk(t)} (C[b,t] . B[b,s]) exp(cs[t] - cs[s]) dt[b,s,h] x[b,s,h,:]
//              + exp(cs[t]) * states[b,chunk(t),h] . C[b,t]  +  D[h] x[b,t,h,:]
//
// Task contract: tasks/mamba2_chunk_scan/reference.py:106-127 (paper listing 1, fp32 decay and
// sums); x [B,L,H,P], dt [B,L,H], dA_cumsum [B,H,NC,CHUNK], Bmat/Cmat [B,L,N], Dskip [H],
// states [B,NC,H,P,N], y [B,L,H,P], all fp16 or bf16, L = NC * CHUNK.
//
// Tensor-core kernel (CHUNK = P = N = 64): one CTA of 256 threads per (two consecutive chunks,
// head, batch); warp w serves the 32 rows (w % 4) * 32 + lane and the 32 columns (w / 4) * 32 + i.  The two chunks are stacked into the 128 rows of one M=128 MMA; every MMA is
// issued twice with half of the accumulator lanes disabled (tcgen05.mma disable-output-lane), so
// a row only ever meets its own chunk's operands:
//   TMA    C rows [128 x 64], x rows [128 s x 64 p], and per chunk c its B rows [64 s x 64 n] and
//          its state tile [64 p x 64 n], stacked as one 256-row operand [B0; St0; B1; St1];
//   MMA    [CB | S] = C . [B0; St0; B1; St1]^T (M=128, N=256, no lane masking): a row of chunk c
//          reads its CB and S from columns [128c, 128c + 64) and [128c + 64, 128c + 128); the other
//          chunk's columns are never read, so nothing of it mixes into the row;
//   rows   w[l,s] = CB[l,s] exp(cs_l - cs_s) dt_s for s <= l else 0, in fp32, written as a
//          16-bit high part and a 16-bit residual (fp16: after a power-of-two row scale that puts
//          the row maximum in [2^14, 2^15), so neither overflow nor underflow loses it);
//   MMA    Yh = Wh . x and Yl = Wl . x (x read MN-major straight from its [s, p] rows);
//   rows   y = (Yh + Yl) / rowscale + exp(cs_l) S + D x, one rounding to 16 bits, 16-byte stores.
//          The residual product is added only where Yh is finite: an infinite x element must give
//          w * inf = +-inf as in the reference, not inf + (residual 0) * inf = NaN.
// A masked entry is an exact zero that still multiplies x (a non-finite x element makes its
// chunk's rows non-finite, as in the reference); specials in states propagate through S.
// Every mbarrier wait is bounded; a timeout is reported through sf_kernel_status.
//
// General kernel (any CHUNK, P, N, alignment): one CTA per (chunk, head, batch) in fp32; W is
// built in shared memory when CHUNK^2 floats fit, else recomputed per output element.
#include "sf_common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <cudaTypedefs.h>
#include <float.h>
#include <atomic>
#include <type_traits>

__device__ sm100::KernelStatus g_mamba2_status;

namespace {

constexpr int CH = 64;                // chunk length, head dim and state dim of the tensor-core kernel
constexpr int ROWS = 2 * CH;          // two chunks per CTA = M of every MMA
constexpr int TILE = ROWS * 128;      // 128 rows of 64 16-bit elements (one 128-byte swizzle row each)
constexpr int HALF = CH * 128;        // 64 such rows
constexpr int NUM_THREADS = 256;
constexpr uint32_t TMEM_COLS = 256;   // [CB0 | S0 | CB1 | S1]; Yh then overwrites [0,64), Yl [128,192)

struct Layout {
    static constexpr int CM = 0;            // C rows, K-major over n
    static constexpr int BS = CM + TILE;    // [B0; St0; B1; St1]: 4 x 64 rows, K-major over n
    static constexpr int X = BS + 2 * TILE; // x rows [s][p]: MN-major B operand of W.x
    static constexpr int WH = X + TILE;     // W high part, K-major over s (row l: its own chunk's s)
    static constexpr int WL = WH + TILE;    // W residual
    static constexpr int CS = WL + TILE;    // float cs[128] * log2(e)
    static constexpr int DT = CS + 512;     // float dt[128]
    static constexpr int MX = DT + 512;     // float row max of |w| over each column half [2][128]
    static constexpr int BARS = MX + 1024;
    static constexpr int BYTES = BARS + 64;
};

struct __align__(8) Bars {
    uint64_t load_full;
    uint64_t cb_full;
    uint64_t y_full;
    uint32_t tmem_base;
};

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

template <typename T>
__device__ __forceinline__ float lo16(uint32_t w) {
    const uint16_t u = (uint16_t)(w & 0xFFFFu);
    return sf::Dt<T>::to_f(*reinterpret_cast<const T*>(&u));
}
template <typename T>
__device__ __forceinline__ float hi16(uint32_t w) {
    const uint16_t u = (uint16_t)(w >> 16);
    return sf::Dt<T>::to_f(*reinterpret_cast<const T*>(&u));
}

// Residual of the 16-bit rounding `hv` of v; zero when hv is not finite (an infinite w must enter
// the product as exactly one infinite term, not inf + nan).
__device__ __forceinline__ float resid(float v, float hv) { return isfinite(hv) ? v - hv : 0.f; }

// Offset of the 16-byte group j (elements 8j..8j+7) of row r in a 128-byte-swizzled tile.
__device__ __forceinline__ int sw128(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

template <typename T>
__global__ void __launch_bounds__(NUM_THREADS, 2)
    mamba2_tc_kernel(const __grid_constant__ CUtensorMap tcm, const __grid_constant__ CUtensorMap tbm,
                     const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tst, const T* __restrict__ dt,
                     const T* __restrict__ cs, const T* __restrict__ dskip, T* __restrict__ y, int L, int H, int NC,
                     sm100::KernelStatus* status) {
    constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + Layout::BARS);
    float* cs_s = reinterpret_cast<float*>(smem + Layout::CS);
    float* dt_s = reinterpret_cast<float*>(smem + Layout::DT);

    float* mx_s = reinterpret_cast<float*>(smem + Layout::MX);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, colh = warp >> 2;  // TMEM lane quarter, column half
    const int pair = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int c0 = 2 * pair;
    const bool has1 = c0 + 1 < NC;
    const int t0 = c0 * CH;
    const int l = quad * 32 + lane, half = l >> 6, ll = l & (CH - 1);
    const bool row_ok = (c0 + half) < NC;

    if (tid == 0) {
        sm100::mbar_init(&bars->load_full, 1);
        sm100::mbar_init(&bars->cb_full, 1);
        sm100::mbar_init(&bars->y_full, 1);
        sm100::fence_mbar_init();
        // Tiles first: their latency overlaps everything up to the first MMA.
        sm100::tma_prefetch_desc(&tcm);
        sm100::tma_prefetch_desc(&tbm);
        sm100::tma_prefetch_desc(&tx);
        sm100::tma_prefetch_desc(&tst);
        sm100::mbar_arrive_expect_tx(&bars->load_full, 2 * TILE + (has1 ? 4 : 2) * HALF);
        sm100::tma_load_3d(smem + Layout::CM, &tcm, &bars->load_full, 0, t0, b);
        for (int c = 0; c < (has1 ? 2 : 1); ++c) {
            sm100::tma_load_3d(smem + Layout::BS + 2 * c * HALF, &tbm, &bars->load_full, 0, t0 + c * CH, b);
            sm100::tma_load_2d(smem + Layout::BS + (2 * c + 1) * HALF, &tst, &bars->load_full, 0,
                               (int)((((int64_t)b * NC + c0 + c) * H + h) * CH));
        }
        sm100::tma_load_3d(smem + Layout::X, &tx, &bars->load_full, h * CH, t0, b);
    }
    if (warp == 0) {
        sm100::tmem_alloc(&bars->tmem_base, TMEM_COLS);
        sm100::tmem_relinquish();
    }
    // Per-row scalars (zero for a missing second chunk): cs * log2(e) by the first 128 threads,
    // dt by the other 128.
    if (colh == 0)
        cs_s[l] = row_ok ? sf::Dt<T>::to_f(cs[(((int64_t)b * H + h) * NC + c0 + half) * CH + ll]) * 1.4426950408889634f : 0.f;
    else
        dt_s[l] = row_ok ? sf::Dt<T>::to_f(dt[((int64_t)b * L + t0 + l) * H + h]) : 0.f;
    const float dh = sf::Dt<T>::to_f(dskip[h]);
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;

    // Lanes of chunk 0 are rows [0,64), of chunk 1 rows [64,128): disable the other half.
    const uint32_t only0[4] = {0u, 0u, 0xFFFFFFFFu, 0xFFFFFFFFu};
    const uint32_t only1[4] = {0xFFFFFFFFu, 0xFFFFFFFFu, 0u, 0u};

    if (tid == 0 && sm100::mbar_wait(&bars->load_full, 0, status, 61)) {
        sm100::tc_fence_after();
        constexpr uint32_t idesc = sm100::idesc_f16(ROWS, 4 * CH, BF16);
        const uint32_t scm = sm100::smem_u32(smem + Layout::CM);
        const uint32_t sbs = sm100::smem_u32(smem + Layout::BS);
#pragma unroll
        for (int k = 0; k < CH / 16; ++k)
            sm100::mma_f16(tmem, sm100::smem_desc_k_sw128(scm + (uint32_t)(k * 32)), sm100::smem_desc_k_sw128(sbs + (uint32_t)(k * 32)), idesc,
                           k > 0 ? 1u : 0u);
        sm100::mma_commit(&bars->cb_full);
    }

    // ---- W: thread (l, colh) builds w[l, s] for its 32 columns s ----
    bool ok = sm100::mbar_wait(&bars->cb_full, 0, status, 62);
    float w[32];
    if (ok) {
        sm100::tc_fence_after();
        uint32_t cb[32];
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)(128 * half + colh * 32), cb);
        sm100::tmem_ld_wait();
        const float csl = cs_s[l];
        const float* csc = cs_s + half * CH + colh * 32;
        const float* dtc = dt_s + half * CH + colh * 32;
        float m = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            w[i] = colh * 32 + i <= ll ? __uint_as_float(cb[i]) * exp2f(csl - csc[i]) * dtc[i] : 0.f;
            m = fmaxf(m, fabsf(w[i]));
        }
        if (!BF16) mx_s[colh * ROWS + l] = m;
    }
    __syncthreads();
    float rinv = 1.f;
    if (ok) {
        float rs = 1.f;
        if (!BF16) {
            const float m = fmaxf(mx_s[l], mx_s[ROWS + l]);
            if (m > 0.f && m <= FLT_MAX) {
                // Power-of-two scale putting the row maximum into [2^14, 2^15).
                int e = (int)((__float_as_uint(m) >> 23) & 0xFFu);
                if (e == 0) e = 1;
                int sx = 141 - e;
                sx = sx > 126 ? 126 : sx;
                rs = __uint_as_float((uint32_t)(sx + 127) << 23);
                rinv = __uint_as_float((uint32_t)(127 - sx) << 23);
            }
        }
        uint8_t* wh = smem + Layout::WH;
        uint8_t* wl = smem + Layout::WL;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = w[j * 8 + i] * rs;
            const uint4 hv = make_uint4(pack2<T>(v[0], v[1]), pack2<T>(v[2], v[3]), pack2<T>(v[4], v[5]), pack2<T>(v[6], v[7]));
            const uint4 lv = make_uint4(pack2<T>(resid(v[0], lo16<T>(hv.x)), resid(v[1], hi16<T>(hv.x))),
                                        pack2<T>(resid(v[2], lo16<T>(hv.y)), resid(v[3], hi16<T>(hv.y))),
                                        pack2<T>(resid(v[4], lo16<T>(hv.z)), resid(v[5], hi16<T>(hv.z))),
                                        pack2<T>(resid(v[6], lo16<T>(hv.w)), resid(v[7], hi16<T>(hv.w))));
            *reinterpret_cast<uint4*>(wh + sw128(l, colh * 4 + j)) = hv;
            *reinterpret_cast<uint4*>(wl + sw128(l, colh * 4 + j)) = lv;
        }
    }
    sm100::fence_proxy_async_smem();
    sm100::tc_fence_before();
    __syncthreads();

    if (tid == 0 && ok) {
        sm100::tc_fence_after();
        constexpr uint32_t idesc = sm100::idesc_f16_bmn(ROWS, CH, BF16);
        const uint32_t sx = sm100::smem_u32(smem + Layout::X);
        const uint32_t wparts[2] = {sm100::smem_u32(smem + Layout::WH), sm100::smem_u32(smem + Layout::WL)};
        for (int q = 0; q < (has1 ? 2 : 1); ++q) {
            const uint32_t(&mask)[4] = q == 0 ? only0 : only1;
            for (int part = 0; part < 2; ++part) {
#pragma unroll
                for (int k = 0; k < CH / 16; ++k) {
                    const uint64_t ad = sm100::smem_desc_k_sw128(wparts[part] + (uint32_t)(k * 32));
                    const uint64_t bd = sm100::smem_desc_mn_sw128(sx + (uint32_t)(q * HALF + k * 16 * 128), TILE, 1024);
                    sm100::mma_f16_lanes(tmem + 128 * part, ad, bd, idesc, k > 0 ? 1u : 0u, mask);
                }
            }
        }
        sm100::mma_commit(&bars->y_full);
    }

    // ---- epilogue: y = (Yh + Yl) / rowscale + exp(cs_l) S + D x for the thread's 32 columns ----
    ok = ok && sm100::mbar_wait(&bars->y_full, 0, status, 63);
    if (ok) {
        sm100::tc_fence_after();
        uint32_t yh[32], yl[32], sr[32];
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)(colh * 32), yh);
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + 128 + (uint32_t)(colh * 32), yl);
        sm100::tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)(128 * half + 64 + colh * 32), sr);
        sm100::tmem_ld_wait();
        if (row_ok) {
            const float ecs = exp2f(cs_s[l]);
            const uint8_t* xs = smem + Layout::X;
            uint4* dst = reinterpret_cast<uint4*>(y + (((int64_t)b * L + t0 + l) * H + h) * CH) + colh * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint4 xv = *reinterpret_cast<const uint4*>(xs + sw128(l, colh * 4 + j));
                const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
                uint32_t o[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float v[2];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int c = j * 8 + 2 * i + e;
                        const float hv = __uint_as_float(yh[c]);
                        const float wx = isfinite(hv) ? hv + __uint_as_float(yl[c]) : hv;
                        const float xe = e ? hi16<T>(xw[i]) : lo16<T>(xw[i]);
                        v[e] = wx * rinv + ecs * __uint_as_float(sr[c]) + dh * xe;
                    }
                    o[i] = pack2<T>(v[0], v[1]);
                }
                dst[j] = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 0) sm100::tmem_dealloc(tmem, TMEM_COLS);
}

// ---- general kernel: fp32, any CHUNK / P / N / alignment ------------------------------------
template <typename T>
__global__ void __launch_bounds__(256)
    mamba2_general_kernel(const T* __restrict__ x, const T* __restrict__ dt, const T* __restrict__ cs, const T* __restrict__ bm,
                          const T* __restrict__ cm, const T* __restrict__ dskip, const T* __restrict__ states, T* __restrict__ y,
                          int64_t L, int64_t H, int64_t P, int64_t N, int64_t C, int64_t NC, bool w_in_smem) {
    extern __shared__ float wsm[];  // [C][C] when w_in_smem
    const int64_t c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const T* csr = cs + ((b * H + h) * NC + c) * C;
    const int64_t r0 = b * L + c * C;  // first row of the chunk in [B*L]
    auto w_at = [&](int64_t l, int64_t s) -> float {
        if (s > l) return 0.f;
        float cb = 0.f;
        for (int64_t n = 0; n < N; ++n) cb += sf::Dt<T>::to_f(cm[(r0 + l) * N + n]) * sf::Dt<T>::to_f(bm[(r0 + s) * N + n]);
        return cb * expf(sf::Dt<T>::to_f(csr[l]) - sf::Dt<T>::to_f(csr[s])) * sf::Dt<T>::to_f(dt[(r0 + s) * H + h]);
    };
    if (w_in_smem) {
        for (int64_t i = threadIdx.x; i < C * C; i += blockDim.x) wsm[i] = w_at(i / C, i % C);
        __syncthreads();
    }
    const float dh = sf::Dt<T>::to_f(dskip[h]);
    const T* st = states + ((b * NC + c) * H + h) * P * N;
    for (int64_t i = threadIdx.x; i < C * P; i += blockDim.x) {
        const int64_t l = i / P, p = i % P;
        float acc = 0.f;
        for (int64_t s = 0; s < C; ++s) {
            const float wv = w_in_smem ? wsm[l * C + s] : w_at(l, s);
            acc += wv * sf::Dt<T>::to_f(x[((r0 + s) * H + h) * P + p]);
        }
        float sv = 0.f;
        for (int64_t n = 0; n < N; ++n) sv += sf::Dt<T>::to_f(cm[(r0 + l) * N + n]) * sf::Dt<T>::to_f(st[p * N + n]);
        const float xv = sf::Dt<T>::to_f(x[((r0 + l) * H + h) * P + p]);
        y[((r0 + l) * H + h) * P + p] = sf::Dt<T>::from_f(acc + expf(sf::Dt<T>::to_f(csr[l])) * sv + dh * xv);
    }
}

sm100::KernelStatus* status_ptr() {
    sm100::KernelStatus* p = nullptr;
    if (cudaGetSymbolAddress((void**)&p, g_mamba2_status) != cudaSuccess) return nullptr;
    return p;
}

template <typename T>
int launch_tc(const void* x, const void* dt, const void* cs, const void* bm, const void* cm, const void* dskip, const void* states,
              void* y, int64_t B, int64_t L, int64_t H, int64_t NC, cudaStream_t st, char* err, uint64_t cap) {
    const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    CUtensorMap mc, mb, mx, ms;
    int rc = sf::tmap_3d(&mc, cm, CH, L, B, CH * 2, L * CH * 2, 64, ROWS, 1, bf16, err, cap);
    if (!rc) rc = sf::tmap_3d(&mb, bm, CH, L, B, CH * 2, L * CH * 2, 64, CH, 1, bf16, err, cap);
    if (!rc) rc = sf::tmap_3d(&mx, x, H * CH, L, B, H * CH * 2, L * H * CH * 2, 64, ROWS, 1, bf16, err, cap);
    if (!rc) rc = sf::tmap_2d(&ms, states, B * NC * H * CH, CH, CH * 2, 64, CH, 2, bf16, err, cap);
    if (rc) return rc;
    sm100::KernelStatus* status = status_ptr();
    if (!status) return sf::fail(SF_EDEVICE, err, cap, "mamba2_chunk_scan: cannot resolve the status word");
    const int smem = Layout::BYTES + 1024;
    static std::atomic<uint64_t> attr_done{0};
    if (sf::once_per_device(attr_done))
        cudaFuncSetAttribute(mamba2_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    const dim3 grid((unsigned)((NC + 1) / 2), (unsigned)H, (unsigned)B);
    mamba2_tc_kernel<T><<<grid, NUM_THREADS, smem, st>>>(mc, mb, mx, ms, (const T*)dt, (const T*)cs, (const T*)dskip, (T*)y, (int)L,
                                                         (int)H, (int)NC, status);
    return sf::check_launch("mamba2_chunk_scan launch", err, cap);
}

template <typename T>
int launch_t(const void* x, const void* dt, const void* cs, const void* bm, const void* cm, const void* dskip, const void* states,
             void* y, int64_t B, int64_t L, int64_t H, int64_t P, int64_t N, int64_t C, int32_t variant, cudaStream_t st, char* err,
             uint64_t cap) {
    const int64_t NC = L / C;
    const bool tc = C == CH && P == CH && N == CH && sf::aligned16(x) && sf::aligned16(bm) && sf::aligned16(cm) &&
                    sf::aligned16(states) && sf::aligned16(y) && B <= 65535 && H <= 65535 && L < (1LL << 31) &&
                    B * NC * H * CH < (1LL << 31);
    if (variant == 1 && !tc)
        return sf::fail(SF_EINVAL, err, cap, "mamba2_chunk_scan: the tensor-core variant needs CHUNK = P = N = 64 and aligned tensors");
    if (tc && variant != 2) return launch_tc<T>(x, dt, cs, bm, cm, dskip, states, y, B, L, H, NC, st, err, cap);
    if (B > 65535 || H > 65535 || NC > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "mamba2_chunk_scan: grid too large");
    const int64_t wbytes = C * C * 4;
    const bool w_in_smem = wbytes <= 96 * 1024;
    static std::atomic<uint64_t> attr_done{0};
    if (sf::once_per_device(attr_done))
        cudaFuncSetAttribute(mamba2_general_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    mamba2_general_kernel<T><<<dim3((unsigned)NC, (unsigned)H, (unsigned)B), 256, w_in_smem ? (size_t)wbytes : 0, st>>>(
        (const T*)x, (const T*)dt, (const T*)cs, (const T*)bm, (const T*)cm, (const T*)dskip, (const T*)states, (T*)y, L, H, P, N, C,
        NC, w_in_smem);
    return sf::check_launch("mamba2_chunk_scan general launch", err, cap);
}

}  // namespace

int sf_mamba2_launch(const void* x, const void* dt, const void* cs, const void* bm, const void* cm, const void* dskip, const void* states,
                     void* y, int64_t B, int64_t L, int64_t H, int64_t P, int64_t N, int64_t C, int32_t dtype, int32_t variant,
                     cudaStream_t st, char* err, uint64_t cap) {
    if (B < 0 || L < 0 || H < 0 || P < 1 || N < 1 || C < 1) return sf::fail(SF_EINVAL, err, cap, "mamba2_chunk_scan: bad sizes");
    if (L % C) return sf::fail(SF_EINVAL, err, cap, "mamba2_chunk_scan: SEQLEN %lld is not a multiple of CHUNK %lld", (long long)L, (long long)C);
    if (B * L * H == 0) return SF_OK;
    if (!x || !dt || !cs || !bm || !cm || !dskip || !states || !y) return sf::fail(SF_EINVAL, err, cap, "mamba2_chunk_scan: null tensor pointer");
    if (dtype == SF_DTYPE_F16) return launch_t<__half>(x, dt, cs, bm, cm, dskip, states, y, B, L, H, P, N, C, variant, st, err, cap);
    if (dtype == SF_DTYPE_BF16) return launch_t<__nv_bfloat16>(x, dt, cs, bm, cm, dskip, states, y, B, L, H, P, N, C, variant, st, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "mamba2_chunk_scan: dtype %d is not fp16/bf16", dtype);
}

int sf_mamba2_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream) {
    sm100::KernelStatus h{0, 0};
    if (cudaMemcpyFromSymbolAsync(&h, g_mamba2_status, sizeof(h), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess) return SF_EDEVICE;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return SF_EDEVICE;
    if (h.code) {
        const sm100::KernelStatus zero{0, 0};
        cudaMemcpyToSymbolAsync(g_mamba2_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream);
        cudaStreamSynchronize(stream);
    }
    *code = h.code;
    *where = h.where;
    return SF_OK;
}

extern "C" int sf_mamba2_chunk_scan(const void* x, const void* dt, const void* dA_cumsum, const void* Bmat, const void* Cmat,
                                    const void* Dskip, const void* states, void* y, int64_t B, int64_t L, int64_t H, int64_t P,
                                    int64_t N, int64_t chunk, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_mamba2_launch(x, dt, dA_cumsum, Bmat, Cmat, Dskip, states, y, B, L, H, P, N, chunk, dtype, 0, (cudaStream_t)stream, err,
                            cap);
}
