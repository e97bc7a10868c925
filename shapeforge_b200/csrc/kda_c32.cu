// Gated delta rule (the gated KDA workload) forward on sm_100a, 32 tokens per chunk, D = 128.
//
// One CTA per (sequence, head) chain.  Per chunk of C = 32 tokens starting from state S0 (fp32,
// [Dv = 128 rows v, Dk = 128 columns c], in TMEM for the whole chain), with b_t the cumulative
// log-decay from the chunk start (per channel), Kp_t = k_t e^{b_t}, Qp_t = q~_t e^{b_t} (q~ = q *
// scale), Kend_t = k_t e^{b_31 - b_t}, A[t,i] = sum_c k_t k_i e^{b_t - b_i} (i < t),
// M[t,i] = sum_c q~_t k_i e^{b_t - b_i} (i <= t), T = (I + diag(beta) A)^-1 diag(beta):
//   w_t = (T V)_t - S0 (T Kp)_t        o_t = (M T V)_t + S0 (Qp - M T Kp)_t
//   S  <- S0 diag(e^{b_31}) + sum_t w_t Kend_t^T
// (the token recurrence of tasks/varlen_kda/reference.py:352-368 with the log-decay supplied,
// summed over the chunk).
//
// Roles (384 threads):
//   warps 0-3   state: thread = value row v.  Lane 0 of warp 0 issues the chain's MMAs:
//               ACC[v, 0:64] = V^T [T ; MT]^T (16-bit high + low parts of T and MT, V MN-major) +
//               S0 . [-K2 ; Q2]^T (tf32, S0 read from TMEM), so ACC holds w^T | o^T directly;
//               after the epilogue and the decay, S += W^T Kend (W as 16-bit high + low parts).
//               The warpgroup stores o, writes W^T (high | low) for that MMA, and decays S in TMEM
//               (S <- S diag(e^{b_31})) once the chunk's first MMA has read it.
//   warps 4-11  prep (thread = channel c x token half), one chunk ahead of the chain: stage q, k,
//               g with cp.async; cumulative decays; the factors of A and M; A | M as one M=64 tf32
//               MMA; T and M T on CUDA cores (16 x 16 blocks); K2 | M T Kp as one bf16x3 MMA
//               (Kp^T MN-major high/low x [T ; MT] high/low); the chain operands.
// A and M are products of per-token factors e^{+-(b_t - r)} with r the midpoint of the channel's
// b range over the chunk: no factor exceeds e^80 while that range stays within 160.  A chunk with
// a wider range (decays below about -5 per token on average) forms A and M pair by pair from
// e^{b_t - b_i} <= 1 instead; per-token decays are floored at -200 (e^-200 is 0 in fp32).  Kp, Qp
// and Kend are exponentials of differences <= 0 for decays <= 0.
// Descriptors of successive K steps are the base descriptor plus the step's byte offset >> 4 (the
// start-address field; shared-memory addresses stay below 2^18, so the field never carries).
// Every mbarrier wait is bounded and reports through sf_kernel_status; a role whose wait gave up
// keeps executing the same barrier sequence without work, so the CTA always runs to its end.
#include "kda_layout.cuh"
#include "sf_common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <atomic>
#include <type_traits>

__device__ sm100::KernelStatus g_kda32_status;

namespace {

constexpr int D = 128;
constexpr int C = 32;
constexpr int NT = 384;
constexpr int NPREP = 256;
constexpr float FACTOR_LIMIT = 80.f;
constexpr float DECAY_FLOOR = -200.f;
// TMEM columns: the state, the w | o accumulator, A | M (M=64 layout), K2 | M T Kp.
constexpr uint32_t TM_S = 0, TM_ACC = 128, TM_D1 = 192, TM_D4 = 256, TMEM_COLS = 512;

struct L {
    static constexpr int B1 = 0;          // [-K2 ; Q2] fp32 K-major: 4 K-blocks x (64 rows x 128 B)
    static constexpr int KE = 32768;      // Kend 16-bit MN-major: 2 x (32 rows x 128 B)
    static constexpr int VB = 40960;      // V 16-bit MN-major, 2 buffers x 2 x (32 x 128 B)
    static constexpr int TMB = 57344;     // [T ; MT] high | low, 16-bit K-major rows of 128 B: 2 buffers x 64 rows
    static constexpr int WT = 73728;      // [W_hi | W_lo]^T K-major rows of 128 B: 128 rows
    static constexpr int SQ = 90112;      // staged q: 2 x (32 x 128 B)
    static constexpr int SK = 98304;      // staged k
    static constexpr int SG = 106496;     // staged g fp32: 4 x (32 x 128 B); b after the factor pass
    static constexpr int PA = 122880;     // [Kf ; Qf] fp32 K-major 4 x (64 x 128 B); then Kp^T high / low
    static constexpr int PB = 155648;     // Kn fp32 K-major 4 x (32 x 128 B)
    static constexpr int TA = 172032;     // A [32][33] fp32
    static constexpr int TMM = 176256;    // M [32][33]
    static constexpr int TT = 180480;     // L^-1, then T [32][33]
    static constexpr int TMT = 184704;    // M T [32][33]
    static constexpr int TP = 188928;     // off-diagonal block product [16][17]
    static constexpr int EL = 190080;     // e^{b_31} [128]
    static constexpr int BS = 190592;     // beta (0 for tokens past the end) [2 buffers][32]
    static constexpr int XTOT = 190848;   // per-channel exchange: b_15, b_31, lo[2], hi[2]
    static constexpr int XLAST = XTOT + 512;
    static constexpr int XLO = XLAST + 512;
    static constexpr int XHI = XLO + 1024;
    static constexpr int VOTE = XHI + 1024;  // 8 words
    static constexpr int OS = 194560;     // o of a chunk [32 t][128 v] 16-bit, written out with 16-byte stores
    static constexpr int BARS = OS + 8192;
    static constexpr int BYTES = BARS + 128;
};
static_assert(L::B1 % 1024 == 0 && L::KE % 1024 == 0 && L::VB % 1024 == 0 && L::TMB % 1024 == 0 && L::WT % 1024 == 0 &&
                  L::SQ % 1024 == 0 && L::SK % 1024 == 0 && L::SG % 1024 == 0 && L::PA % 1024 == 0 && L::PB % 1024 == 0,
              "operand tiles are 1024-byte aligned");

struct __align__(8) Bars {
    uint64_t stg_full;  // staged q, k, g landed (256 cp.async arrivals)
    uint64_t v_full[2]; // V of a chunk landed (256 cp.async arrivals)
    uint64_t p1;        // A | M MMA done (commit)
    uint64_t p4;        // K2 | M T Kp MMA done (commit)
    uint64_t cfull;     // chain operands of the next chunk written (256 prep arrivals)
    uint64_t m1;        // w | o accumulator ready (commit)
    uint64_t wready;    // W^T written and S decayed (128 arrivals)
    uint64_t m2;        // state update done (commit)
    uint32_t tmem_base;
};

using kdal::chunk128;
using kdal::from16;
using kdal::kmaj32;
using kdal::mnmaj16;
using kdal::pack_hi_lo;
using kdal::to16;

// Stage one chunk's q, k (16-bit), g and beta (fp32) into shared memory with cp.async: tokens past
// the chain's end are zero-filled (nothing is read for them).  Every prep thread copies its share
// and arrives on the staging barrier.
template <typename T>
__device__ __forceinline__ void stage_chunk(uint8_t* smem, const T* q, const T* k, const float* g, const float* beta, int buf, int t0,
                                            int nt, int H, int h, int p, uint64_t* bar) {
    const uint32_t base = sm100::smem_u32(smem);
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        const int id = p + NPREP * m;  // 512 chunks of 16 B per 16-bit tensor: (t, j16)
        const int t = id >> 4, j16 = id & 15;
        const bool live = t < nt;
        const size_t row = ((size_t)(t0 + (live ? t : 0)) * H + h) * D + 8 * j16;
        const int off = (j16 >> 3) * 4096 + chunk128(t, j16);
        sm100::cp_async_16(base + L::SQ + off, q + row, live ? 16u : 0u);
        sm100::cp_async_16(base + L::SK + off, k + row, live ? 16u : 0u);
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int id = p + NPREP * m;  // 1024 chunks of 16 B of fp32 g: (t, j32)
        const int t = id >> 5, j = id & 31;
        const bool live = t < nt;
        const size_t row = ((size_t)(t0 + (live ? t : 0)) * H + h) * D + 4 * j;
        sm100::cp_async_16(base + L::SG + (j >> 3) * 4096 + chunk128(t, j), g + row, live ? 16u : 0u);
    }
    if (p < C) {
        const bool live = p < nt;
        sm100::cp_async_4(base + L::BS + 128 * buf + 4 * p, beta + (size_t)(t0 + (live ? p : 0)) * H + h, live ? 4u : 0u);
    }
    sm100::cp_async_mbar_arrive(bar);
}

template <typename T>
__device__ __forceinline__ void stage_v(uint8_t* smem, int buf, const T* v, int t0, int nt, int H, int h, int p, uint64_t* bar) {
    const uint32_t base = sm100::smem_u32(smem) + L::VB + buf * 8192;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
        const int id = p + NPREP * m;
        const int t = id >> 4, j16 = id & 15;
        const bool live = t < nt;
        const size_t row = ((size_t)(t0 + (live ? t : 0)) * H + h) * D + 8 * j16;
        sm100::cp_async_16(base + (j16 >> 3) * 4096 + chunk128(t, j16), v + row, live ? 16u : 0u);
    }
    sm100::cp_async_mbar_arrive(bar);
}

template <typename T>
__global__ void __launch_bounds__(NT, 1)
    kda_c32_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ g,
                   const float* __restrict__ beta, const int32_t* __restrict__ cu, const float* __restrict__ state0, float scale, int H,
                   T* __restrict__ out, float* __restrict__ final_state, sm100::KernelStatus* status) {
    constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + L::BARS);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int chain = blockIdx.x;
    const int s = chain / H, h = chain % H;
    const int begin = cu[s], end = cu[s + 1];
    if (begin < 0 || end < 0 || end < begin) return;  // sentinel: not part of this batch
    const int ntok = end - begin;
    const int nchunks = (ntok + C - 1) / C;

    if (tid == 0) {
        sm100::mbar_init(&bars->stg_full, NPREP);
        sm100::mbar_init(&bars->v_full[0], NPREP);
        sm100::mbar_init(&bars->v_full[1], NPREP);
        sm100::mbar_init(&bars->p1, 1);
        sm100::mbar_init(&bars->p4, 1);
        sm100::mbar_init(&bars->cfull, NPREP);
        sm100::mbar_init(&bars->m1, 1);
        sm100::mbar_init(&bars->wready, 128);
        sm100::mbar_init(&bars->m2, 1);
        sm100::fence_mbar_init();
    }
    if (warp == 0) {
        sm100::tmem_alloc(&bars->tmem_base, TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    bool ok = true;

    if (warp >= 4) {
        // ======================= prep =======================
        const int p = tid - 128;
        const int c = p & 127, half = p >> 7;
        const int pw = p >> 5;  // prep warp 0..7
        const uint32_t lane_q = (uint32_t)((pw & 3) * 32) << 16;
        float* el = reinterpret_cast<float*>(smem + L::EL);
        float* ta = reinterpret_cast<float*>(smem + L::TA);
        float* tmm = reinterpret_cast<float*>(smem + L::TMM);
        float* tt = reinterpret_cast<float*>(smem + L::TT);
        float* tmt = reinterpret_cast<float*>(smem + L::TMT);
        float* tp = reinterpret_cast<float*>(smem + L::TP);
        float* xtot = reinterpret_cast<float*>(smem + L::XTOT);
        float* xlast = reinterpret_cast<float*>(smem + L::XLAST);
        float* xlo = reinterpret_cast<float*>(smem + L::XLO);
        float* xhi = reinterpret_cast<float*>(smem + L::XHI);
        uint32_t* vote = reinterpret_cast<uint32_t*>(smem + L::VOTE);
        uint32_t p1_phase = 0;
        if (nchunks > 0) {
            stage_chunk<T>(smem, q, k, g, beta, 0, begin, min(C, ntok), H, h, p, &bars->stg_full);
            stage_v<T>(smem, 0, v, begin, min(C, ntok), H, h, p, &bars->v_full[0]);
        }
        for (int ci = 0; ci < nchunks; ++ci) {
            const int b = ci & 1;
            const int t0 = begin + ci * C;
            const int nt = min(C, end - t0);
            if (!sm100::mbar_wait(&bars->stg_full, ci & 1, status, 80)) ok = false;
            const float* bs = reinterpret_cast<const float*>(smem + L::BS + 128 * b);

            // ---- factor pass: thread (c, half) covers tokens 16*half .. 16*half + 15 ----
            float bl[16], kv[16], qv[16];
            {
                const float* sg = reinterpret_cast<const float*>(smem + L::SG);
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = 16 * half + j;
                    float gl = *reinterpret_cast<const float*>(smem + L::SG + kmaj32(t, c, 4096));
                    gl = gl < DECAY_FLOOR ? DECAY_FLOOR : gl;  // NaN passes through
                    acc += t < nt ? gl : 0.f;
                    bl[j] = acc;
                    kv[j] = from16<T>(*reinterpret_cast<const uint16_t*>(smem + L::SK + mnmaj16(t, c, 4096)));
                    qv[j] = from16<T>(*reinterpret_cast<const uint16_t*>(smem + L::SQ + mnmaj16(t, c, 4096))) * scale;
                }
                (void)sg;
                if (half == 0) xtot[c] = acc;
            }
            sm100::named_barrier_sync(1, NPREP);
            if (half == 1) {
                const float off = xtot[c];
#pragma unroll
                for (int j = 0; j < 16; ++j) bl[j] += off;
            }
            {
                float lo = bl[0], hi = bl[0];
#pragma unroll
                for (int j = 1; j < 16; ++j) {
                    lo = fminf(lo, bl[j]);
                    hi = fmaxf(hi, bl[j]);
                }
                xlo[half * 128 + c] = lo;
                xhi[half * 128 + c] = hi;
                if (half == 1) xlast[c] = bl[15];
#pragma unroll
                for (int j = 0; j < 16; ++j)  // b over g, for the pairwise path (own elements only)
                    *reinterpret_cast<float*>(smem + L::SG + kmaj32(16 * half + j, c, 4096)) = bl[j];
            }
            sm100::named_barrier_sync(1, NPREP);
            const float blo = fminf(xlo[c], xlo[128 + c]), bhi = fmaxf(xhi[c], xhi[128 + c]);
            const float blast = xlast[c];
            const float ref = 0.5f * (blo + bhi);
            const bool wide = !(0.5f * (bhi - blo) <= FACTOR_LIMIT);  // NaN counts as wide
            {
                const bool any = __any_sync(0xffffffffu, wide);
                if (lane == 0) vote[pw] = any ? 1u : 0u;
            }
            const float elast = __expf(blast);
            const float elr = __expf(blast - ref);
            float kp[16];
            {
                // Kf, Qf (A rows) and Kn (B rows) of the A | M MMA.  Qp seeds the M T Kp columns of
                // the K2 | M T Kp accumulator (the MMA then subtracts M T Kp, giving Q2), whose K2
                // columns start at zero.  A wide channel (only possible when the chunk takes the
                // pairwise path, so Kn is not used) keeps Kend = k e^{b_31 - b} where Kn would be.
                const float er = __expf(ref);
                uint32_t qp[16], zero[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = 16 * half + j;
                    const float x = bl[j] - ref;
                    const float e = __expf(x), en = __expf(-x);
                    const float kf = kv[j] * e, qf = qv[j] * e, kn = kv[j] * en;
                    *reinterpret_cast<float*>(smem + L::PA + kmaj32(t, c, 8192)) = kf;
                    *reinterpret_cast<float*>(smem + L::PA + kmaj32(C + t, c, 8192)) = qf;
                    float qpv;
                    if (!wide) {
                        kp[j] = kf * er;
                        qpv = qf * er;
                        *reinterpret_cast<float*>(smem + L::PB + kmaj32(t, c, 4096)) = kn;
                    } else {
                        const float e0 = __expf(bl[j]);
                        kp[j] = kv[j] * e0;
                        qpv = qv[j] * e0;
                        *reinterpret_cast<float*>(smem + L::PB + kmaj32(t, c, 4096)) = kv[j] * __expf(blast - bl[j]);
                    }
                    qp[j] = __float_as_uint(qpv);
                    zero[j] = 0u;
                }
                sm100::tmem_st_32x32b_x16(tmem + lane_q + TM_D4 + (uint32_t)(16 * half), zero);
                sm100::tmem_st_32x32b_x16(tmem + lane_q + TM_D4 + (uint32_t)(C + 16 * half), qp);
                sm100::tmem_st_wait();
            }
            sm100::tc_fence_before();
            sm100::fence_proxy_async_smem();
            sm100::named_barrier_sync(1, NPREP);
            const bool exact = (vote[0] | vote[1] | vote[2] | vote[3] | vote[4] | vote[5] | vote[6] | vote[7]) != 0u;

            if (!exact) {
                // ---- A | M = [Kf ; Qf] . Kn^T: M = 64, N = 32, K = 128 (tf32) ----
                if (p == 0) {
                    sm100::tc_fence_after();
                    constexpr uint32_t idesc = sm100::idesc_tf32(64, 32);
                    const uint64_t ad0 = sm100::smem_desc_k_sw128(sm100::smem_u32(smem + L::PA));
                    const uint64_t bd0 = sm100::smem_desc_k_sw128(sm100::smem_u32(smem + L::PB));
#pragma unroll
                    for (int kk = 0; kk < D / 8; ++kk)
                        sm100::mma_tf32(tmem + TM_D1, ad0 + (uint64_t)(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4),
                                        bd0 + (uint64_t)(((kk >> 2) * 4096 + (kk & 3) * 32) >> 4), idesc, kk > 0 ? 1u : 0u);
                    sm100::mma_commit(&bars->p1);
                }
                __syncwarp();
                // The staging buffer is free: stage the next chunk while this one is prepared.
                if (ci + 1 < nchunks) stage_chunk<T>(smem, q, k, g, beta, b ^ 1, t0 + C, min(C, end - t0 - C), H, h, p, &bars->stg_full);
                if (!sm100::mbar_wait(&bars->p1, p1_phase & 1, status, 81)) ok = false;
                ++p1_phase;
                sm100::tc_fence_after();
                {
                    // M=64 layout: rows 16*i + r sit in TMEM lane 32*i + r (r < 16).  Quadrant 0/1:
                    // A rows 0-15 / 16-31; quadrant 2/3: M rows 0-15 / 16-31.  Warps 0-3 take
                    // columns 0-15, warps 4-7 columns 16-31.
                    uint32_t r[16];
                    sm100::tmem_ld_32x32b_x16(tmem + lane_q + TM_D1 + (uint32_t)((pw >> 2) * 16), r);
                    sm100::tmem_ld_wait();
                    if (lane < 16) {
                        const int qd = pw & 3;
                        const int t = (qd & 1) * 16 + lane;
                        float* dst = qd < 2 ? ta : tmm;
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int i = (pw >> 2) * 16 + j;
                            const bool keep = qd < 2 ? (i < t) : (i <= t);
                            dst[t * 33 + i] = keep ? __uint_as_float(r[j]) : 0.f;
                        }
                    }
                }
            } else {
                // ---- pairwise A and M (any decay): thread -> row t, columns i0, i0+8, i0+16, i0+24 ----
                const int t = p >> 3, i0 = p & 7;
                const float* bsm = reinterpret_cast<const float*>(smem + L::SG);
                float a[4] = {0.f, 0.f, 0.f, 0.f}, m[4] = {0.f, 0.f, 0.f, 0.f};
                if (t < nt) {
#pragma unroll 2
                    for (int cc = 0; cc < D; ++cc) {
                        const int col = (cc + 4 * i0) & (D - 1);
                        const float bt = *reinterpret_cast<const float*>(smem + L::SG + kmaj32(t, col, 4096));
                        const float kt = from16<T>(*reinterpret_cast<const uint16_t*>(smem + L::SK + mnmaj16(t, col, 4096)));
                        const float qt = from16<T>(*reinterpret_cast<const uint16_t*>(smem + L::SQ + mnmaj16(t, col, 4096)));
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int i = i0 + 8 * u;
                            if (i <= t) {
                                const float bi = *reinterpret_cast<const float*>(smem + L::SG + kmaj32(i, col, 4096));
                                const float ki = from16<T>(*reinterpret_cast<const uint16_t*>(smem + L::SK + mnmaj16(i, col, 4096))) *
                                                 __expf(bt - bi);
                                a[u] = fmaf(kt, ki, a[u]);
                                m[u] = fmaf(qt, ki, m[u]);
                            }
                        }
                    }
                }
                (void)bsm;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int i = i0 + 8 * u;
                    const bool live = t < nt && i < nt;
                    ta[t * 33 + i] = (live && i < t) ? a[u] : 0.f;
                    tmm[t * 33 + i] = (live && i <= t) ? m[u] * scale : 0.f;
                }
                sm100::named_barrier_sync(1, NPREP);
                if (ci + 1 < nchunks) stage_chunk<T>(smem, q, k, g, beta, b ^ 1, t0 + C, min(C, end - t0 - C), H, h, p, &bars->stg_full);
            }
            // -Kp^T (16-bit high and low, MN-major) into the A|M operand space (its MMA is done).
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int t = 16 * half + j;
                const float nk = -kp[j];
                const uint16_t hv = to16<T>(nk);
                const float fh = from16<T>(hv);
                const uint16_t lv = to16<T>(isfinite(fh) ? nk - fh : 0.f);
                *reinterpret_cast<uint16_t*>(smem + L::PA + mnmaj16(t, c, 4096)) = hv;
                *reinterpret_cast<uint16_t*>(smem + L::PA + 8192 + mnmaj16(t, c, 4096)) = lv;
            }
            sm100::named_barrier_sync(1, NPREP);

            // ---- T = (I + diag(beta) A)^-1 diag(beta) in 16 x 16 blocks ----
            if (p < 32) {
                const int bb = p >> 4, j = p & 15, o = 16 * bb;
                float x[16];
#pragma unroll
                for (int r = 0; r < 16; ++r) {
                    float acc = 0.f;
#pragma unroll
                    for (int i = 0; i < r; ++i) acc = fmaf(ta[(o + r) * 33 + o + i], x[i], acc);
                    x[r] = (r == j ? 1.f : 0.f) - bs[o + r] * acc;
                }
#pragma unroll
                for (int r = 0; r < 16; ++r) tt[(o + r) * 33 + o + j] = x[r];
            }
            sm100::named_barrier_sync(1, NPREP);
            {
                // P = diag(beta_2) A21 L11^-1, then L21^-1 = -L22^-1 P; the upper-right block is 0.
                const int r = p >> 4, j = p & 15;
                float acc = 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) acc = fmaf(ta[(16 + r) * 33 + i], tt[i * 33 + j], acc);
                tp[r * 17 + j] = bs[16 + r] * acc;
                tt[r * 33 + 16 + j] = 0.f;
            }
            sm100::named_barrier_sync(1, NPREP);
            {
                const int r = p >> 4, j = p & 15;
                float acc = 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) acc = fmaf(tt[(16 + r) * 33 + 16 + i], tp[i * 17 + j], acc);
                tt[(16 + r) * 33 + j] = -acc;
            }
            sm100::named_barrier_sync(1, NPREP);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = p + NPREP * u, r = e >> 5, j = e & 31;
                tt[r * 33 + j] *= bs[j];
            }
            sm100::named_barrier_sync(1, NPREP);
            {
                // M T: thread -> row r, columns j0, j0+8, j0+16, j0+24.  M and T are stored with
                // zeros above their diagonals, so the full sum over i is the triangular product.
                const int r = p >> 3, j0 = p & 7;
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int i = 0; i < C; ++i) {
                    const float mri = tmm[r * 33 + i];
#pragma unroll
                    for (int u = 0; u < 4; ++u) acc[u] = fmaf(mri, tt[i * 33 + j0 + 8 * u], acc[u]);
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) tmt[r * 33 + j0 + 8 * u] = acc[u];
            }
            sm100::named_barrier_sync(1, NPREP);
            {
                // [T ; MT] as 16-bit high | low rows: thread -> row n, 8 columns.
                const int n = p >> 2, i0 = (p & 3) * 8;
                const float* src = n < C ? tt + n * 33 : tmt + (n - C) * 33;
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) hi[u] = pack_hi_lo<T>(src[i0 + 2 * u], src[i0 + 2 * u + 1], lo[u]);
                uint8_t* row = smem + L::TMB + b * 8192;
                *reinterpret_cast<uint4*>(row + chunk128(n, i0 >> 3)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<uint4*>(row + chunk128(n, 4 + (i0 >> 3))) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
            sm100::fence_proxy_async_smem();
            sm100::named_barrier_sync(1, NPREP);

            // ---- [-K2 | Q2] = [0 | Qp] + (-Kp)^T . [T ; MT]^T: M = 128 (channels), N = 64, K = 32, bf16 x3 ----
            if (p == 0) {
                sm100::tc_fence_after();
                constexpr uint32_t idesc = sm100::idesc_f16_major(128, 64, BF16, true, false);
                const uint64_t ad0 = sm100::smem_desc_mn_sw128(sm100::smem_u32(smem + L::PA), 4096, 1024);
                const uint64_t bd0 = sm100::smem_desc_k_sw128(sm100::smem_u32(smem + L::TMB + b * 8192));
#pragma unroll
                for (int part = 0; part < 3; ++part) {
                    const uint32_t a_part = part == 2 ? 8192u : 0u;   // Kp high, high, low
                    const uint32_t b_part = part == 1 ? 64u : 0u;     // [T ; MT] high, low, high
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk)
                        sm100::mma_f16(tmem + TM_D4, ad0 + (uint64_t)((a_part + kk * 2048) >> 4), bd0 + (uint64_t)((b_part + kk * 32) >> 4),
                                       idesc, 1u);
                }
                sm100::mma_commit(&bars->p4);
            }
            __syncwarp();
            if (!sm100::mbar_wait(&bars->p4, ci & 1, status, 82)) ok = false;
            sm100::tc_fence_after();
            uint32_t k2r[16], q2r[16];
            sm100::tmem_ld_32x32b_x16(tmem + lane_q + TM_D4 + (uint32_t)(16 * half), k2r);
            sm100::tmem_ld_32x32b_x16(tmem + lane_q + TM_D4 + (uint32_t)(C + 16 * half), q2r);
            sm100::tmem_ld_wait();
            sm100::tc_fence_before();

            // ---- hand-off: the chain's previous update has consumed B1 / KE / EL ----
            if (ci > 0 && !sm100::mbar_wait(&bars->m2, (ci - 1) & 1, status, 83)) ok = false;
            if (ci + 1 < nchunks) stage_v<T>(smem, b ^ 1, v, t0 + C, min(C, end - t0 - C), H, h, p, &bars->v_full[b ^ 1]);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int t = 16 * half + j;
                *reinterpret_cast<uint32_t*>(smem + L::B1 + kmaj32(t, c, 8192)) = k2r[j];
                *reinterpret_cast<uint32_t*>(smem + L::B1 + kmaj32(C + t, c, 8192)) = q2r[j];
                const float kn = *reinterpret_cast<const float*>(smem + L::PB + kmaj32(t, c, 4096));
                *reinterpret_cast<uint16_t*>(smem + L::KE + mnmaj16(t, c, 4096)) = to16<T>(wide ? kn : kn * elr);
            }
            if (half == 0) el[c] = elast;
            if (!sm100::mbar_wait(&bars->v_full[b], (ci >> 1) & 1, status, 84)) ok = false;
            sm100::fence_proxy_async_smem();
            sm100::mbar_arrive(&bars->cfull);
        }
        (void)ok;
    } else {
        // ======================= state (value row v = tid) =======================
        const int vr = tid;
        const uint32_t lane_q = (uint32_t)(warp * 32) << 16;
        const size_t srow = (((size_t)s * H + h) * D + vr) * D;
#pragma unroll 1
        for (int cb = 0; cb < 4; ++cb) {
            uint32_t r[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(state0 ? state0[srow + cb * 32 + j] : 0.f);
            sm100::tmem_st_32x32b_x32(tmem + lane_q + TM_S + (uint32_t)(cb * 32), r);
        }
        sm100::tmem_st_wait();
        sm100::tc_fence_before();
        sm100::named_barrier_sync(2, 128);
        sm100::tc_fence_after();
        const float* el = reinterpret_cast<const float*>(smem + L::EL);
        for (int ci = 0; ci < nchunks; ++ci) {
            const int b = ci & 1;
            const int t0 = begin + ci * C;
            const int nt = min(C, end - t0);
            if (tid == 0) {
                if (!sm100::mbar_wait(&bars->cfull, ci & 1, status, 85)) ok = false;
                sm100::tc_fence_after();
                if (ok) {
                    constexpr uint32_t idv = sm100::idesc_f16_major(128, 64, BF16, true, false);
                    const uint64_t vd0 = sm100::smem_desc_mn_sw128(sm100::smem_u32(smem + L::VB + b * 8192), 4096, 1024);
                    const uint64_t td0 = sm100::smem_desc_k_sw128(sm100::smem_u32(smem + L::TMB + b * 8192));
#pragma unroll
                    for (int part = 0; part < 2; ++part) {
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk)
                            sm100::mma_f16(tmem + TM_ACC, vd0 + (uint64_t)((kk * 2048) >> 4), td0 + (uint64_t)((part * 64 + kk * 32) >> 4),
                                           idv, (part | kk) != 0 ? 1u : 0u);
                    }
                    constexpr uint32_t idt = sm100::idesc_tf32(128, 64);
                    const uint64_t b1d = sm100::smem_desc_k_sw128(sm100::smem_u32(smem + L::B1));
#pragma unroll
                    for (int kk = 0; kk < D / 8; ++kk)
                        sm100::mma_tf32_ta(tmem + TM_ACC, tmem + TM_S + (uint32_t)(kk * 8), b1d + (uint64_t)(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4),
                                           idt, 1u);
                }
                sm100::mma_commit(&bars->m1);
            }
            __syncwarp();
            if (!sm100::mbar_wait(&bars->cfull, ci & 1, status, 88)) ok = false;  // e^{b_31} of this chunk written
            if (!sm100::mbar_wait(&bars->m1, ci & 1, status, 86)) ok = false;
            sm100::tc_fence_after();
            uint32_t wr[32], orr[32];
            sm100::tmem_ld_32x32b_x32(tmem + lane_q + TM_ACC, wr);
            sm100::tmem_ld_32x32b_x32(tmem + lane_q + TM_ACC + C, orr);
            sm100::tmem_ld_wait();
            {
                // o^T row v -> o [t][v] in shared memory, then whole 256-byte token rows to global
                // with 16-byte stores (rows past the chain's end are not stored).
                uint16_t* os = reinterpret_cast<uint16_t*>(smem + L::OS);
#pragma unroll
                for (int t = 0; t < C; ++t) os[t * D + vr] = to16<T>(__uint_as_float(orr[t]));
                sm100::named_barrier_sync(3, 128);
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const int id = vr + 128 * m, t = id >> 4, j = id & 15;
                    if (t < nt)
                        *reinterpret_cast<uint4*>(out + ((size_t)(t0 + t) * H + h) * D + 8 * j) =
                            *reinterpret_cast<const uint4*>(smem + L::OS + t * 256 + 16 * j);
                }
                sm100::named_barrier_sync(3, 128);
            }
            {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) hi[u] = pack_hi_lo<T>(__uint_as_float(wr[2 * u]), __uint_as_float(wr[2 * u + 1]), lo[u]);
                uint8_t* row = smem + L::WT;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    *reinterpret_cast<uint4*>(row + chunk128(vr, j)) = make_uint4(hi[4 * j], hi[4 * j + 1], hi[4 * j + 2], hi[4 * j + 3]);
                    *reinterpret_cast<uint4*>(row + chunk128(vr, 4 + j)) = make_uint4(lo[4 * j], lo[4 * j + 1], lo[4 * j + 2], lo[4 * j + 3]);
                }
            }
            // S <- S diag(e^{b_31}) (the chunk's first MMA has read S; cfull made e^{b_31} visible).
#pragma unroll 1
            for (int cb = 0; cb < 4; ++cb) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem + lane_q + TM_S + (uint32_t)(cb * 32), r);
                sm100::tmem_ld_wait();
                const float4* e4 = reinterpret_cast<const float4*>(el + cb * 32);
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 e = e4[j4];
                    r[4 * j4] = __float_as_uint(__uint_as_float(r[4 * j4]) * e.x);
                    r[4 * j4 + 1] = __float_as_uint(__uint_as_float(r[4 * j4 + 1]) * e.y);
                    r[4 * j4 + 2] = __float_as_uint(__uint_as_float(r[4 * j4 + 2]) * e.z);
                    r[4 * j4 + 3] = __float_as_uint(__uint_as_float(r[4 * j4 + 3]) * e.w);
                }
                sm100::tmem_st_32x32b_x32(tmem + lane_q + TM_S + (uint32_t)(cb * 32), r);
            }
            sm100::tmem_st_wait();
            sm100::fence_proxy_async_smem();
            sm100::tc_fence_before();
            sm100::mbar_arrive(&bars->wready);
            if (tid == 0) {
                if (!sm100::mbar_wait(&bars->wready, ci & 1, status, 87)) ok = false;
                sm100::tc_fence_after();
                if (ok) {
                    constexpr uint32_t idu = sm100::idesc_f16_bmn(128, D, BF16);
                    const uint64_t wd0 = sm100::smem_desc_k_sw128(sm100::smem_u32(smem + L::WT));
                    const uint64_t kd0 = sm100::smem_desc_mn_sw128(sm100::smem_u32(smem + L::KE), 4096, 1024);
#pragma unroll
                    for (int part = 0; part < 2; ++part) {
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk)
                            sm100::mma_f16(tmem + TM_S, wd0 + (uint64_t)((part * 64 + kk * 32) >> 4), kd0 + (uint64_t)((kk * 2048) >> 4), idu, 1u);
                    }
                }
                sm100::mma_commit(&bars->m2);
            }
            __syncwarp();
        }
        // ---- final state ----
        if (nchunks > 0 && !sm100::mbar_wait(&bars->m2, (nchunks - 1) & 1, status, 90)) ok = false;
        sm100::tc_fence_after();
        if (ok) {
#pragma unroll 1
            for (int cb = 0; cb < 4; ++cb) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem + lane_q + TM_S + (uint32_t)(cb * 32), r);
                sm100::tmem_ld_wait();
                float4* dst = reinterpret_cast<float4*>(final_state + srow + cb * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                                         __uint_as_float(r[4 * j + 3]));
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 0) sm100::tmem_dealloc(tmem, TMEM_COLS);
}

sm100::KernelStatus* status_ptr() {
    sm100::KernelStatus* p = nullptr;
    if (cudaGetSymbolAddress((void**)&p, g_kda32_status) != cudaSuccess) return nullptr;
    return p;
}

}  // namespace

// The 32-token chunked kernel for D = 128 with 16-byte-aligned q/k/v/g rows; returns SF_EINVAL
// (without launching) when the shape or alignment does not qualify.
int sf_kda_gated_c32_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                            const void* initial_state, void* out, void* final_state, int64_t N, int64_t H, int64_t Dd, float scale,
                            int32_t dtype, cudaStream_t st, char* err, uint64_t cap) {
    if (Dd != D || !sf::aligned16(q) || !sf::aligned16(k) || !sf::aligned16(v) || !sf::aligned16(g) || !sf::aligned16(final_state) ||
        (initial_state && !sf::aligned16(initial_state)))
        return sf::fail(SF_EINVAL, err, cap, "kda: the 32-token chunked kernel needs D = 128 and 16-byte-aligned tensors");
    if (N * H > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "kda: too many chains");
    sm100::KernelStatus* status = status_ptr();
    if (!status) return sf::fail(SF_EDEVICE, err, cap, "kda: cannot resolve the status word");
    const int smem = L::BYTES + 1024;
    static std::atomic<uint64_t> attr_done{0};
    if (sf::once_per_device(attr_done)) {
        cudaFuncSetAttribute(kda_c32_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        cudaFuncSetAttribute(kda_c32_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    }
    if (dtype == SF_DTYPE_F16)
        kda_c32_kernel<__half><<<(unsigned)(N * H), NT, smem, st>>>((const __half*)q, (const __half*)k, (const __half*)v, (const float*)g,
                                                                    (const float*)beta, (const int32_t*)cu_seqlens,
                                                                    (const float*)initial_state, scale, (int)H, (__half*)out,
                                                                    (float*)final_state, status);
    else
        kda_c32_kernel<__nv_bfloat16><<<(unsigned)(N * H), NT, smem, st>>>(
            (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (const float*)g, (const float*)beta,
            (const int32_t*)cu_seqlens, (const float*)initial_state, scale, (int)H, (__nv_bfloat16*)out, (float*)final_state, status);
    return sf::check_launch("kda_gated c32 launch", err, cap);
}

int sf_kda32_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream) {
    sm100::KernelStatus hs{0, 0};
    if (cudaMemcpyFromSymbolAsync(&hs, g_kda32_status, sizeof(hs), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess) return SF_EDEVICE;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return SF_EDEVICE;
    if (hs.code) {
        const sm100::KernelStatus zero{0, 0};
        cudaMemcpyToSymbolAsync(g_kda32_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream);
        cudaStreamSynchronize(stream);
    }
    *code = hs.code;
    *where = hs.where;
    return SF_OK;
}
