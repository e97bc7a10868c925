// Chunked gated delta rule (KDA) forward on the tcgen05 tensor cores, sm_100a, D = 128.
//
// Per (sequence, head) chain the recurrence of kda.cu is evaluated 16 tokens at a time.  With
// b_t = sum_{i<=t} g_i (per key channel, cumulative log-decay inside the chunk), the state after
// token t of a chunk that starts from S0 is
//   S_t = S0 diag(e^{b_t}) + sum_{i<=t} w_i (k_i * e^{b_t - b_i})^T
// where the rows w_i [Dv] solve the unit lower-triangular system
//   w_t = beta_t (v_t - S0 (k_t * e^{b_t}) - sum_{i<t} A[t,i] w_i),  A[t,i] = <k_t e^{b_t}, k_i e^{-b_i}>
// and the outputs are
//   o_t = S0 (q~_t * e^{b_t}) + sum_{i<=t} M[t,i] w_i,               M[t,i] = <q~_t e^{b_t}, k_i e^{-b_i}>
// (q~ = q * scale); the chunk ends with S = S0 diag(e^{b_15}) + W^T Kend, Kend_i = k_i e^{b_15 - b_i}.
// Every exponential the kernel takes is finite for any log-decay: A and M are products of factors
// e^{+-(b_t - r)} measured from a per-channel reference r at the midpoint of that channel's b range
// over the chunk (no factor above e^80 while the range stays within 160, i.e. decays above about
// -10 per token on average), and a chunk with a wider range forms A and M pair by pair from
// e^{b_t - b_i} <= 1; Kp, Qp and Kend are exponentials of b_t, b_15 - b_t <= 0.  Per-token decays
// are floored at -200 (e^-200 is 0 in fp32 either way).
//
// Writing B = diag(beta) and T = (I + B A)^-1 B (16 x 16, lower triangular, state-independent),
// the rows of a chunk are
//   w = T (V - U'),  U'_t = S0 Kp_t     =>   w_t = Vt_t - S0 K2_t,          Vt = T V,  K2 = T Kp
//   o_t = S0 Qp_t + (M w)_t             =>   o_t = Ov_t + S0 Q2_t,          Ov = (M T) V,  Q2 = Qp - (M T) Kp
// so everything the state chain needs besides S0 is prepared ahead.
//
// One CTA of 384 threads per chain; the 128 x 128 fp32 state lives in TMEM (lane = value row v,
// column = key channel k) and is never written to memory until the chain ends.  Warpgroups 1 and 2
// (prep) take the even and the odd chunks and run up to two chunks ahead of warpgroup 0 (state),
// each through its own chunk buffer:
//   prep   thread = key channel: cumulative decay, the factored keys/queries in fp32, the 16 x 16
//          A and M products, T by forward substitution and M T, all in the warpgroup's own
//          scratch; only then does it wait for its chunk buffer to be released and write Kend
//          (16-bit, the update MMA's operand), K2 and Q2 (fp32, the tf32 MMA operand), T, M T, v and
//          the chunk decay e^{b_15}; the next chunk's inputs are loaded into registers meanwhile;
//   state  MMA 1  [W' | O'] = S0 . [-K2 ; Q2]^T as tf32 with S0 read straight from TMEM as the A
//          operand (M=128 rows v, N=32, K=128); while it runs, thread = value row computes
//          Vt = T v and Ov = (M T) v for its row;
//          then w = Vt + (-W'), o = Ov + O' (fp32), outputs stored, w written as a 16-bit high part
//          and residual, S0 decayed in TMEM (S0 diag(e^{b_15}));
//          MMA 2  S += W^T . Kend (high and residual parts; M=128, N=128, K=16), whose completion
//          also hands the chunk's buffers back to the prep warpgroup.  The next chunk's MMA 1 is
//          issued behind it: the tensor pipe runs one CTA's MMAs in issue order.
// The task op (tasks/varlen_kda/reference.py:323-374) runs the same kernel with TASK = true: g and beta
// arrive as 16-bit tensors, each chunk's q and k rows are L2-normalised (rsqrt(sum x^2 + 1e-6), q times
// the scale tensor) from the staged registers, the log-decay is LOWER_BOUND * sigmoid(exp(A_log[h]) *
// (g + dt_bias[h, c])) (in [LOWER_BOUND, 0] per token) and beta is sigmoid(beta).
// Every mbarrier wait is bounded; a timeout is reported through sf_kernel_status.
#include "sf_common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <atomic>
#include <type_traits>

__device__ sm100::KernelStatus g_kda_status;

namespace {

constexpr int D = 128;       // head dim (key and value)
constexpr int C = 16;        // tokens per chunk
constexpr int NT = 384;      // threads: a state warpgroup and two prep warpgroups
constexpr int WG = 128;      // threads per warpgroup
constexpr int KP = D + 4;    // fp32 staging row stride: 16-byte rows, rows r and r+8 in distinct bank groups
constexpr uint32_t TMEM_COLS = 256;  // S [0,128), [W'|O'] [128,160)
// A and M are formed from per-token factors e^{+-(b_t - r)}, r the midpoint of a channel's b range
// over the chunk; a channel whose half-range exceeds this could overflow them (e^88 is fp32's
// limit), and the chunk then takes the pairwise path.
constexpr float FACTOR_LIMIT = 80.f;
// Per-token log-decays are floored here: e^-200 is 0 in fp32 either way, and the floor keeps the
// cumulative sums, and the differences of them that the kernel exponentiates, precise.
constexpr float DECAY_FLOOR = -200.f;

struct Layout {
    static constexpr int WH = 0;                   // W^T high [128 v x 64 (t < 16 used)], 16-bit K-major
    static constexpr int WL = WH + 16384;          // W^T residual
    // Chunk buffers (x2, one per prep warpgroup), released by the update MMA's commit.
    static constexpr int B1 = WL + 16384;          // [-K2 ; Q2] fp32 [32 x 128] K-major, 4 K-blocks x 4 KB
    static constexpr int B1_BYTES = 16384;
    static constexpr int KE = B1 + 2 * B1_BYTES;   // Kend [16 t x 128 k] 16-bit MN-major, 2 blocks x 2 KB
    static constexpr int VB = KE + 2 * 4096;       // v (16-bit) [16][128]
    static constexpr int TB = VB + 2 * C * D * 2;  // T [16][16] then M T [16][16], fp32
    static constexpr int EB = TB + 2 * 2 * C * C * 4;  // fp32 chunk decay e^{b_15} [128]
    // Per prep warpgroup scratch: fp32 [16][KP] Kp, Kn, Qp; staged q, k, v (16-bit), g (fp32), beta;
    // the 16 x 16 fp32 A, M, T and M T.
    static constexpr int PREP = EB + 2 * D * 4;
    static constexpr int KP32 = 0;
    static constexpr int KN32 = KP32 + C * KP * 4;
    static constexpr int QP32 = KN32 + C * KP * 4;
    static constexpr int QS = QP32 + C * KP * 4;
    static constexpr int KS = QS + C * D * 2;
    static constexpr int VS = KS + C * D * 2;
    static constexpr int GS = VS + C * D * 2;
    static constexpr int BS = GS + C * D * 4;
    static constexpr int TA = BS + 64;
    static constexpr int TM = TA + C * C * 4;
    static constexpr int TT = TM + C * C * 4;
    static constexpr int TMT = TT + C * C * 4;
    static constexpr int NQ = TMT + C * C * 4;     // task: inverse L2 norms of q and k per token
    static constexpr int NK = NQ + C * 4;
    static constexpr int WIDE = NK + C * 4;        // per-warp votes: a channel's decay range is too wide to factor
    static constexpr int PREP_BYTES = WIDE + 16;
    static constexpr int BARS = PREP + 2 * PREP_BYTES;
    static constexpr int BYTES = BARS + 64;
};
static_assert(Layout::B1 % 1024 == 0 && Layout::KE % 1024 == 0, "MMA operands need 1024-byte alignment");
static_assert(Layout::PREP % 16 == 0 && Layout::PREP_BYTES % 16 == 0, "16-byte staging rows");

struct __align__(8) Bars {
    uint64_t m1;
    uint64_t m2;
    uint64_t pfull[2];   // prep -> state: chunk buffers ready (128 arrivals)
    uint64_t pempty[2];  // state -> prep: chunk buffers consumed (the update MMA's commit)
    uint32_t tmem_base;
};

template <typename T>
__device__ __forceinline__ uint16_t to16(float x) {
    const T h = sf::Dt<T>::from_f(x);
    return *reinterpret_cast<const uint16_t*>(&h);
}
template <typename T>
__device__ __forceinline__ float from16(uint16_t u) {
    return sf::Dt<T>::to_f(*reinterpret_cast<const T*>(&u));
}

// Byte offset of 16-bit element (row r, column c) of a 128-byte-swizzled operand whose blocks of
// 64 columns are `blk` bytes apart.
__device__ __forceinline__ int kmaj(int r, int c, int blk) {
    return (c >> 6) * blk + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + ((c & 7) << 1);
}

// Byte offset of fp32 element (row r, column c) of a K-major 128-byte-swizzled operand with K-blocks
// of 32 columns, 32 rows (4 KB) each.
__device__ __forceinline__ int kmaj32(int r, int c) {
    return (c >> 5) * 4096 + r * 128 + ((((c & 31) >> 2) ^ (r & 7)) << 4) + ((c & 3) << 2);
}

// Packed fp32 pair FMA (one FFMA2 for two lanes of work).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(reinterpret_cast<uint64_t&>(d))
        : "l"(reinterpret_cast<const uint64_t&>(a)), "l"(reinterpret_cast<const uint64_t&>(b)), "l"(reinterpret_cast<const uint64_t&>(c)));
    return d;
}

// Next chunk's raw inputs, held in registers while the current chunk computes.  Thread tid covers
// token tid / 8 and the 16 columns (tid % 8) * 16 .. +15.
struct Prefetch {
    uint4 q[2], k[2], v[2];
    float4 g[4];   // gated: fp32 log-decay
    uint4 g16[2];  // task: 16-bit g
    float beta;
};

// Task inputs that the gated workload does not have.
struct TaskArgs {
    const float* a_log;    // [H]
    const float* dt_bias;  // [H * D]
    const float* scale;    // [1]
    float lower_bound;
};

template <typename T, bool TASK>
__device__ __forceinline__ void load_chunk(Prefetch& p, const T* q, const T* k, const T* v, const void* g, const void* beta, int t0,
                                           int nt, int H, int h, int tid) {
    const int tt = tid >> 3, part = tid & 7;
    const bool live = tt < nt;
    const size_t base = ((size_t)(t0 + tt) * H + h) * D + part * 16;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        p.q[i] = live ? __ldg(reinterpret_cast<const uint4*>(q + base) + i) : make_uint4(0, 0, 0, 0);
        p.k[i] = live ? __ldg(reinterpret_cast<const uint4*>(k + base) + i) : make_uint4(0, 0, 0, 0);
        p.v[i] = live ? __ldg(reinterpret_cast<const uint4*>(v + base) + i) : make_uint4(0, 0, 0, 0);
    }
    if (TASK) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
            p.g16[i] = live ? __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(g) + base) + i) : make_uint4(0, 0, 0, 0);
        p.beta = (tid < nt) ? sf::Dt<T>::to_f(reinterpret_cast<const T*>(beta)[(size_t)(t0 + tid) * H + h]) : -INFINITY;  // sigmoid -> 0
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i)
            p.g[i] = live ? __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(g) + base) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        p.beta = (tid < nt) ? __ldg(reinterpret_cast<const float*>(beta) + (size_t)(t0 + tid) * H + h) : 0.f;
    }
}

template <typename T>
__device__ __forceinline__ float sum_sq16(const uint4 (&w)[2]) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t r[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = from16<T>((uint16_t)(r[j] & 0xFFFFu)), b = from16<T>((uint16_t)(r[j] >> 16));
            s = fmaf(a, a, fmaf(b, b, s));
        }
    }
    return s;
}

// Staged chunk -> the prep warpgroup's scratch.  Task: g converted to fp32, sigmoid(beta), and the
// inverse L2 norms of each token's q and k rows (the 8 threads of a token reduce by shuffles).
template <typename T, bool TASK>
__device__ __forceinline__ void store_chunk(const Prefetch& p, uint8_t* prep, int tid) {
    const int tt = tid >> 3, part = tid & 7;
    const int off = (tt * D + part * 16) * 2;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        *reinterpret_cast<uint4*>(prep + Layout::QS + off + 16 * i) = p.q[i];
        *reinterpret_cast<uint4*>(prep + Layout::KS + off + 16 * i) = p.k[i];
        *reinterpret_cast<uint4*>(prep + Layout::VS + off + 16 * i) = p.v[i];
    }
    float* gs = reinterpret_cast<float*>(prep + Layout::GS) + tt * D + part * 16;
    if (TASK) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint32_t r[4] = {p.g16[i].x, p.g16[i].y, p.g16[i].z, p.g16[i].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                gs[8 * i + 2 * j] = from16<T>((uint16_t)(r[j] & 0xFFFFu));
                gs[8 * i + 2 * j + 1] = from16<T>((uint16_t)(r[j] >> 16));
            }
        }
        float sq = sum_sq16<T>(p.q), sk = sum_sq16<T>(p.k);
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
            sk += __shfl_xor_sync(0xffffffffu, sk, o);
        }
        if (part == 0) {
            reinterpret_cast<float*>(prep + Layout::NQ)[tt] = rsqrtf(sq + 1e-6f);
            reinterpret_cast<float*>(prep + Layout::NK)[tt] = rsqrtf(sk + 1e-6f);
        }
        if (tid < C) reinterpret_cast<float*>(prep + Layout::BS)[tid] = 1.0f / (1.0f + __expf(-p.beta));
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) reinterpret_cast<float4*>(gs)[i] = p.g[i];
        if (tid < C) reinterpret_cast<float*>(prep + Layout::BS)[tid] = p.beta;
    }
}

template <typename T, bool TASK>
__global__ void __launch_bounds__(NT, 1)
    kda_chunk_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const void* __restrict__ g,
                     const void* __restrict__ beta, const int32_t* __restrict__ cu, const float* __restrict__ state0, float scale,
                     int H, T* __restrict__ out, float* __restrict__ final_state, sm100::KernelStatus* status, TaskArgs task) {
    constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + Layout::BARS);
    float* eb = reinterpret_cast<float*>(smem + Layout::EB);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int wg = warp >> 2, wtid = tid & (WG - 1);
    const int chain = blockIdx.x;
    const int s = chain / H, h = chain % H;
    const int begin = cu[s], end = cu[s + 1];
    if (begin < 0 || end < 0 || end < begin) return;  // sentinel: not part of this batch

    if (tid == 0) {
        sm100::mbar_init(&bars->m1, 1);
        sm100::mbar_init(&bars->m2, 1);
        for (int b = 0; b < 2; ++b) {
            sm100::mbar_init(&bars->pfull[b], WG);
            sm100::mbar_init(&bars->pempty[b], 1);
        }
        sm100::fence_mbar_init();
    }
    if (warp == 0) {
        sm100::tmem_alloc(&bars->tmem_base, TMEM_COLS);
        sm100::tmem_relinquish();
    }
    const int nchunks = (end - begin + C - 1) / C;
    Prefetch pf;
    const int pw = wg - 1;  // prep warpgroup index (chunks pw, pw + 2, ...; buffer pw)
    if (wg >= 1 && pw < nchunks) load_chunk<T, TASK>(pf, q, k, v, g, beta, begin + pw * C, min(C, end - begin - pw * C), H, h, wtid);
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const int vrow = wtid;  // value row owned by a state thread (TMEM lane)
    const size_t srow = (((size_t)s * H + h) * D + vrow) * D;
    bool ok = true;

    if (wg >= 1) {
        // ================= prep warpgroups =================
        uint8_t* prep = smem + Layout::PREP + pw * Layout::PREP_BYTES;
        float* kp32 = reinterpret_cast<float*>(prep + Layout::KP32);
        float* kn32 = reinterpret_cast<float*>(prep + Layout::KN32);
        float* qp32 = reinterpret_cast<float*>(prep + Layout::QP32);
        float* ta = reinterpret_cast<float*>(prep + Layout::TA);
        float* tm = reinterpret_cast<float*>(prep + Layout::TM);
        float* tt = reinterpret_cast<float*>(prep + Layout::TT);
        float* tmt = reinterpret_cast<float*>(prep + Layout::TMT);
        const float* bs = reinterpret_cast<const float*>(prep + Layout::BS);
        const uint32_t bar_id = 1 + 2 * pw;
        const int b = pw;
        const int c = wtid;  // key channel (and value channel)
        // Task gate constants of this channel; the q scale (a tensor for the task op).
        const float task_ea = TASK ? __expf(task.a_log[h]) : 0.f;
        const float task_dtb = TASK ? task.dt_bias[(size_t)h * D + c] : 0.f;
        const float task_lb = TASK ? task.lower_bound : 0.f;
        const float qscale = TASK ? *task.scale : scale;
        for (int ci = pw; ci < nchunks && ok; ci += 2) {
            const int t0 = begin + ci * C;
            const int nt_chunk = min(C, end - t0);  // tokens past the sequence end contribute no decay
            sm100::named_barrier_sync(bar_id, WG);  // previous iteration's reads of the prep scratch are done
            store_chunk<T, TASK>(pf, prep, wtid);
            sm100::named_barrier_sync(bar_id, WG);
            if (ci + 2 < nchunks) load_chunk<T, TASK>(pf, q, k, v, g, beta, t0 + 2 * C, min(C, end - t0 - 2 * C), H, h, wtid);

            // ---- factors in fp32 (thread = key channel c) ----
            // b_t = the cumulative log-decay from the chunk start.  A and M need e^{b_t - b_i}
            // (i <= t); they are products of per-token factors e^{+-(b_t - r)} measured from this
            // channel's reference r, the midpoint of its b range over the chunk, so no factor is
            // larger than e^{half-range}.  When any channel's half-range exceeds FACTOR_LIMIT the
            // chunk forms A and M pair by pair instead (exact for any decay).  Kp, Qp (measured
            // from the chunk start) and Kend (to the chunk end) are exponentials of differences
            // that are <= 0 for decays <= 0, and stay finite for every input.
            float kp[C], qp[C];
            float elast;
            bool exact;
            {
                float* gs = reinterpret_cast<float*>(prep + Layout::GS);
                const uint16_t* ks = reinterpret_cast<const uint16_t*>(prep + Layout::KS);
                const uint16_t* qs = reinterpret_cast<const uint16_t*>(prep + Layout::QS);
                float bcum[C];
                float bacc = 0.f, blo = 0.f, bhi = 0.f;
#pragma unroll
                for (int t = 0; t < C; ++t) {
                    float gl = gs[t * D + c];
                    if (TASK) gl = task_lb * (1.0f / (1.0f + __expf(-task_ea * (gl + task_dtb))));
                    gl = gl < DECAY_FLOOR ? DECAY_FLOOR : gl;  // NaN passes through
                    bacc += t < nt_chunk ? gl : 0.f;
                    bcum[t] = bacc;
                    blo = t == 0 ? bacc : fminf(blo, bacc);
                    bhi = t == 0 ? bacc : fmaxf(bhi, bacc);
                    gs[t * D + c] = bacc;  // b, for the pairwise path and Kend (own column only)
                }
                elast = __expf(bacc);
                const float ref = 0.5f * (blo + bhi);
                const bool wide = !(0.5f * (bhi - blo) <= FACTOR_LIMIT);  // NaN counts as wide
                const bool warp_wide = __any_sync(0xffffffffu, wide);
                if ((wtid & 31) == 0) reinterpret_cast<uint32_t*>(prep + Layout::WIDE)[wtid >> 5] = warp_wide ? 1u : 0u;
                const float* nq = reinterpret_cast<const float*>(prep + Layout::NQ);
                const float* nk = reinterpret_cast<const float*>(prep + Layout::NK);
#pragma unroll
                for (int t = 0; t < C; ++t) {
                    const float kv = from16<T>(ks[t * D + c]) * (TASK ? nk[t] : 1.0f);
                    const float qv = from16<T>(qs[t * D + c]) * (TASK ? nq[t] * qscale : qscale);
                    const float x = bcum[t] - ref;
                    const float e = __expf(x), en = __expf(-x), e0 = __expf(bcum[t]);
                    kp[t] = kv * e0;
                    qp[t] = qv * e0;
                    kp32[t * KP + c] = kv * e;
                    kn32[t * KP + c] = kv * en;
                    qp32[t * KP + c] = qv * e;
                }
            }
            sm100::named_barrier_sync(bar_id, WG);
            {
                const uint32_t* votes = reinterpret_cast<const uint32_t*>(prep + Layout::WIDE);
                exact = (votes[0] | votes[1] | votes[2] | votes[3]) != 0u;
            }
            if (!exact) {
                // A[t][i] (i < t) and M[t][i] (i <= t): thread -> rows t of Kp and Qp, columns i and
                // i + 8; even and odd channels accumulate in the two halves of packed pairs.
                const int t = wtid >> 3, i0c = wtid & 7;
                const float4* lk = reinterpret_cast<const float4*>(kp32 + t * KP);
                const float4* lq = reinterpret_cast<const float4*>(qp32 + t * KP);
                const float4* r0 = reinterpret_cast<const float4*>(kn32 + i0c * KP);
                const float4* r1 = reinterpret_cast<const float4*>(kn32 + (i0c + 8) * KP);
                float2 a0 = make_float2(0.f, 0.f), a1 = a0, m0 = a0, m1 = a0;
#pragma unroll 2
                for (int cc = 0; cc < D / 4; ++cc) {
                    const float4 x = lk[cc], y = lq[cc], u = r0[cc], w = r1[cc];
                    a0 = ffma2(make_float2(x.x, x.y), make_float2(u.x, u.y), a0);
                    a0 = ffma2(make_float2(x.z, x.w), make_float2(u.z, u.w), a0);
                    a1 = ffma2(make_float2(x.x, x.y), make_float2(w.x, w.y), a1);
                    a1 = ffma2(make_float2(x.z, x.w), make_float2(w.z, w.w), a1);
                    m0 = ffma2(make_float2(y.x, y.y), make_float2(u.x, u.y), m0);
                    m0 = ffma2(make_float2(y.z, y.w), make_float2(u.z, u.w), m0);
                    m1 = ffma2(make_float2(y.x, y.y), make_float2(w.x, w.y), m1);
                    m1 = ffma2(make_float2(y.z, y.w), make_float2(w.z, w.w), m1);
                }
                ta[t * C + i0c] = i0c < t ? a0.x + a0.y : 0.f;
                ta[t * C + i0c + 8] = i0c + 8 < t ? a1.x + a1.y : 0.f;
                tm[t * C + i0c] = i0c <= t ? m0.x + m0.y : 0.f;
                tm[t * C + i0c + 8] = i0c + 8 <= t ? m1.x + m1.y : 0.f;
            } else {
                // Pairwise: A[t][i] = sum_c k_t k_i e^{b_t - b_i}, M[t][i] = sum_c q~_t k_i e^{b_t - b_i},
                // one exponential per (pair, channel).  Columns are visited from a per-thread offset
                // so the eight rows i of a warp fall in distinct banks.
                const int t = wtid >> 3, i0c = wtid & 7;
                const float* bs32 = reinterpret_cast<const float*>(prep + Layout::GS);
                const uint16_t* ks = reinterpret_cast<const uint16_t*>(prep + Layout::KS);
                const uint16_t* qs = reinterpret_cast<const uint16_t*>(prep + Layout::QS);
                const float* nq = reinterpret_cast<const float*>(prep + Layout::NQ);
                const float* nk = reinterpret_cast<const float*>(prep + Layout::NK);
                const float nkt = TASK ? nk[t] : 1.0f, nqt = TASK ? nq[t] * qscale : qscale;
#pragma unroll 1
                for (int half = 0; half < 2; ++half) {
                    const int i = i0c + 8 * half;
                    float a = 0.f, m = 0.f;
                    if (i <= t) {
#pragma unroll 4
                        for (int cc = 0; cc < D; ++cc) {
                            const int col = (cc + 4 * i0c) & (D - 1);
                            const float ki = from16<T>(ks[i * D + col]) * __expf(bs32[t * D + col] - bs32[i * D + col]);
                            a = fmaf(from16<T>(ks[t * D + col]), ki, a);
                            m = fmaf(from16<T>(qs[t * D + col]), ki, m);
                        }
                    }
                    const float nki = TASK ? nk[i] : 1.0f;
                    ta[t * C + i] = i < t ? a * nkt * nki : 0.f;
                    tm[t * C + i] = i <= t ? m * nqt * nki : 0.f;
                }
            }
            sm100::named_barrier_sync(bar_id, WG);
            {
                // Kend_t = k_t e^{b_15 - b_t} into this channel's column of Kn (A and M are done with it).
                const float* bs32 = reinterpret_cast<const float*>(prep + Layout::GS);
                const uint16_t* ks = reinterpret_cast<const uint16_t*>(prep + Layout::KS);
                const float* nk = reinterpret_cast<const float*>(prep + Layout::NK);
                const float blast = bs32[(C - 1) * D + c];
#pragma unroll
                for (int t = 0; t < C; ++t)
                    kn32[t * KP + c] = from16<T>(ks[t * D + c]) * (TASK ? nk[t] : 1.0f) * __expf(blast - bs32[t * D + c]);
            }
            if (wtid < C) {
                // T = (I + B A)^-1 B, column j by forward substitution: x_t = [t == j] - beta_t sum_{i<t} A[t][i] x_i.
                const int j = wtid;
                float x[C];
#pragma unroll
                for (int t = 0; t < C; ++t) {
                    float acc = 0.f;
#pragma unroll
                    for (int i = 0; i < t; ++i) acc = fmaf(ta[t * C + i], x[i], acc);
                    x[t] = (t == j ? 1.f : 0.f) - bs[t] * acc;
                }
                const float bj = bs[j];
#pragma unroll
                for (int t = 0; t < C; ++t) tt[t * C + j] = x[t] * bj;
            }
            sm100::named_barrier_sync(bar_id, WG);
            {
                // M T (lower triangular): thread -> row t, columns jc and jc + 8.
                const int t = wtid >> 3, jc = wtid & 7;
                float s0 = 0.f, s1 = 0.f;
#pragma unroll
                for (int i = 0; i < C; ++i) {
                    const float mi = tm[t * C + i];
                    s0 = fmaf(mi, tt[i * C + jc], s0);
                    s1 = fmaf(mi, tt[i * C + jc + 8], s1);
                }
                tmt[t * C + jc] = s0;
                tmt[t * C + jc + 8] = s1;
            }
            sm100::named_barrier_sync(bar_id, WG);

            // ---- the chunk buffer: released by the update MMA of chunk ci - 2 ----
            if (ci >= 2 && !sm100::mbar_wait(&bars->pempty[b], ((ci >> 1) - 1) & 1, status, 74)) {
                ok = false;
                break;
            }
            {
                uint8_t* b1 = smem + Layout::B1 + b * Layout::B1_BYTES;
                uint8_t* keb = smem + Layout::KE + b * 4096;
                eb[b * D + c] = elast;
                // -K2 = -T Kp and Q2 = Qp - (M T) Kp (rows t and 16 + t of the tf32 MMA operand).
#pragma unroll
                for (int t = 0; t < C; ++t) {
                    float k2 = 0.f, q2 = qp[t];
#pragma unroll
                    for (int i = 0; i <= t; ++i) {
                        k2 = fmaf(-tt[t * C + i], kp[i], k2);
                        q2 = fmaf(-tmt[t * C + i], kp[i], q2);
                    }
                    *reinterpret_cast<float*>(b1 + kmaj32(t, c)) = k2;
                    *reinterpret_cast<float*>(b1 + kmaj32(C + t, c)) = q2;
                    *reinterpret_cast<uint16_t*>(keb + kmaj(t, c, 2048)) = to16<T>(kn32[t * KP + c]);  // Kend = k e^{b_15 - b_t}
                }
                // T, M T and v for the state warpgroup's Vt = T v, Ov = (M T) v.
                float* tb = reinterpret_cast<float*>(smem + Layout::TB) + b * 2 * C * C;
                reinterpret_cast<float4*>(tb)[wtid] = wtid < 64 ? reinterpret_cast<const float4*>(tt)[wtid]
                                                                 : reinterpret_cast<const float4*>(tmt)[wtid - 64];
                const uint4* vsrc = reinterpret_cast<const uint4*>(prep + Layout::VS);
                uint4* vdst = reinterpret_cast<uint4*>(smem + Layout::VB + b * C * D * 2);
                vdst[wtid] = vsrc[wtid];
                vdst[wtid + WG] = vsrc[wtid + WG];
            }
            sm100::fence_proxy_async_smem();  // B1 / KE are read by the MMAs
            sm100::mbar_arrive(&bars->pfull[b]);
        }
    } else {
        // ================= state warpgroup =================
        // Initial state -> TMEM (zero when none is given).
#pragma unroll 1
        for (int cb = 0; cb < 4; ++cb) {
            uint32_t r[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(state0 ? state0[srow + cb * 32 + j] : 0.f);
            sm100::tmem_st_32x32b_x32(tmem + lane_off + (uint32_t)(cb * 32), r);
        }
        sm100::tmem_st_wait();
        sm100::tc_fence_before();
        sm100::named_barrier_sync(2, WG);
        for (int ci = 0; ci < nchunks && ok; ++ci) {
            const int b = ci & 1;
            const int t0 = begin + ci * C;
            const int nt = min(C, end - t0);
            if (!sm100::mbar_wait(&bars->pfull[b], (ci >> 1) & 1, status, 75)) {
                ok = false;
                break;
            }
            // ---- MMA 1: [-W' | O'] = S0 . [-K2 ; Q2]^T, tf32, S0 from TMEM.  Issued behind the
            // previous chunk's update MMA, which the tensor pipe completes first. ----
            if (wtid == 0) {
                sm100::tc_fence_after();
                constexpr uint32_t idesc = sm100::idesc_tf32(128, 2 * C);
                const uint32_t sb = sm100::smem_u32(smem + Layout::B1 + b * Layout::B1_BYTES);
#pragma unroll
                for (int kk = 0; kk < D / 8; ++kk) {
                    const uint64_t bd = sm100::smem_desc_k_sw128(sb + (uint32_t)((kk >> 2) * 4096 + (kk & 3) * 32));
                    sm100::mma_tf32_ta(tmem + 128, tmem + (uint32_t)(kk * 8), bd, idesc, kk > 0 ? 1u : 0u);
                }
                sm100::mma_commit(&bars->m1);
            }
            // ---- while MMA 1 runs: Vt = T v and Ov = (M T) v for this value row ----
            float vt[C], ov[C];
            {
                const float* tb = reinterpret_cast<const float*>(smem + Layout::TB) + b * 2 * C * C;
                const uint16_t* vb = reinterpret_cast<const uint16_t*>(smem + Layout::VB + b * C * D * 2);
                float vv[C];
#pragma unroll
                for (int i = 0; i < C; ++i) vv[i] = from16<T>(vb[i * D + vrow]);
#pragma unroll
                for (int t = 0; t < C; ++t) {
                    float a = 0.f, o = 0.f;
#pragma unroll
                    for (int i = 0; i <= t; ++i) {
                        a = fmaf(tb[t * C + i], vv[i], a);
                        o = fmaf(tb[C * C + t * C + i], vv[i], o);
                    }
                    vt[t] = a;
                    ov[t] = o;
                }
            }
            if (!sm100::mbar_wait(&bars->m1, ci & 1, status, 72)) {
                ok = false;
                break;
            }
            sm100::tc_fence_after();

            // ---- rows: w = Vt - W', o = Ov + O'; S0 decayed in TMEM ----
            {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem + lane_off + 128, r);
                sm100::tmem_ld_wait();
                float w[C];
#pragma unroll
                for (int t = 0; t < C; ++t) {
                    w[t] = vt[t] + __uint_as_float(r[t]);
                    const float o = ov[t] + __uint_as_float(r[C + t]);
                    if (t < nt) out[((size_t)(t0 + t) * H + h) * D + vrow] = sf::Dt<T>::from_f(o);
                }
                // W^T row v: t = 0..15 is K of the update MMA (16-byte groups 0 and 1 of the row).
                uint32_t hi[8], lo[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint16_t h0 = to16<T>(w[2 * j]), h1 = to16<T>(w[2 * j + 1]);
                    const float f0 = from16<T>(h0), f1 = from16<T>(h1);
                    hi[j] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                    const float r0 = isfinite(f0) ? w[2 * j] - f0 : 0.f, r1 = isfinite(f1) ? w[2 * j + 1] - f1 : 0.f;
                    lo[j] = (uint32_t)to16<T>(r0) | ((uint32_t)to16<T>(r1) << 16);
                }
#pragma unroll
                for (int grp = 0; grp < 2; ++grp) {
                    const int off = vrow * 128 + ((grp ^ (vrow & 7)) << 4);
                    *reinterpret_cast<uint4*>(smem + Layout::WH + off) = make_uint4(hi[4 * grp], hi[4 * grp + 1], hi[4 * grp + 2], hi[4 * grp + 3]);
                    *reinterpret_cast<uint4*>(smem + Layout::WL + off) = make_uint4(lo[4 * grp], lo[4 * grp + 1], lo[4 * grp + 2], lo[4 * grp + 3]);
                }
            }
            {
                const float4* e4 = reinterpret_cast<const float4*>(eb + b * D);
#pragma unroll 1
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t r[2][32];
#pragma unroll
                    for (int c2 = 0; c2 < 2; ++c2) sm100::tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)((2 * hh + c2) * 32), r[c2]);
                    sm100::tmem_ld_wait();
#pragma unroll
                    for (int c2 = 0; c2 < 2; ++c2) {
                        const int cb = 2 * hh + c2;
#pragma unroll
                        for (int j4 = 0; j4 < 8; ++j4) {
                            const float4 e = e4[cb * 8 + j4];
                            r[c2][4 * j4] = __float_as_uint(__uint_as_float(r[c2][4 * j4]) * e.x);
                            r[c2][4 * j4 + 1] = __float_as_uint(__uint_as_float(r[c2][4 * j4 + 1]) * e.y);
                            r[c2][4 * j4 + 2] = __float_as_uint(__uint_as_float(r[c2][4 * j4 + 2]) * e.z);
                            r[c2][4 * j4 + 3] = __float_as_uint(__uint_as_float(r[c2][4 * j4 + 3]) * e.w);
                        }
                        sm100::tmem_st_32x32b_x32(tmem + lane_off + (uint32_t)(cb * 32), r[c2]);
                    }
                }
                sm100::tmem_st_wait();
            }
            sm100::fence_proxy_async_smem();
            sm100::tc_fence_before();
            sm100::named_barrier_sync(2, WG);

            // ---- MMA 2: S += W^T . Kend (high + residual); its completion frees buffer b ----
            if (wtid == 0) {
                sm100::tc_fence_after();
                constexpr uint32_t idesc = sm100::idesc_f16_bmn(128, D, BF16);
                const uint64_t bd = sm100::smem_desc_mn_sw128(sm100::smem_u32(smem + Layout::KE + b * 4096), 2048, 1024);
                sm100::mma_f16(tmem, sm100::smem_desc_k_sw128(sm100::smem_u32(smem + Layout::WH)), bd, idesc, 1u);
                sm100::mma_f16(tmem, sm100::smem_desc_k_sw128(sm100::smem_u32(smem + Layout::WL)), bd, idesc, 1u);
                sm100::mma_commit(&bars->m2);
                sm100::mma_commit(&bars->pempty[b]);
            }
        }
    }

    // ---- final state (state warpgroup) ----
    if (wg == 0 && ok && nchunks > 0 && !sm100::mbar_wait(&bars->m2, (nchunks - 1) & 1, status, 73)) ok = false;
    sm100::tc_fence_after();
    if (wg == 0 && ok) {
#pragma unroll 1
        for (int cb = 0; cb < 4; ++cb) {
            uint32_t r[32];
            sm100::tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)(cb * 32), r);
            sm100::tmem_ld_wait();
            float4* dst = reinterpret_cast<float4*>(final_state + srow + cb * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                                     __uint_as_float(r[4 * j + 3]));
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 0) sm100::tmem_dealloc(tmem, TMEM_COLS);
}

sm100::KernelStatus* status_ptr() {
    sm100::KernelStatus* p = nullptr;
    if (cudaGetSymbolAddress((void**)&p, g_kda_status) != cudaSuccess) return nullptr;
    return p;
}

}  // namespace

namespace {

template <bool TASK>
int chunk_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                 const void* initial_state, void* out, void* final_state, int64_t N, int64_t H, int64_t Dd, float scale, TaskArgs task,
                 int32_t dtype, cudaStream_t st, char* err, uint64_t cap) {
    if (Dd != D || !sf::aligned16(q) || !sf::aligned16(k) || !sf::aligned16(v) || !sf::aligned16(g) || !sf::aligned16(final_state) ||
        (initial_state && !sf::aligned16(initial_state)))
        return sf::fail(SF_EINVAL, err, cap, "kda: the chunked kernel needs D = 128 and 16-byte-aligned tensors");
    if (N * H > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "kda: too many chains");
    sm100::KernelStatus* status = status_ptr();
    if (!status) return sf::fail(SF_EDEVICE, err, cap, "kda: cannot resolve the status word");
    const int smem = Layout::BYTES + 1024;
    static std::atomic<uint64_t> attr_done{0};
    if (sf::once_per_device(attr_done)) {
        cudaFuncSetAttribute(kda_chunk_kernel<__half, TASK>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        cudaFuncSetAttribute(kda_chunk_kernel<__nv_bfloat16, TASK>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    }
    if (dtype == SF_DTYPE_F16)
        kda_chunk_kernel<__half, TASK><<<(unsigned)(N * H), NT, smem, st>>>(
            (const __half*)q, (const __half*)k, (const __half*)v, g, beta, (const int32_t*)cu_seqlens, (const float*)initial_state, scale,
            (int)H, (__half*)out, (float*)final_state, status, task);
    else
        kda_chunk_kernel<__nv_bfloat16, TASK><<<(unsigned)(N * H), NT, smem, st>>>(
            (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta, (const int32_t*)cu_seqlens,
            (const float*)initial_state, scale, (int)H, (__nv_bfloat16*)out, (float*)final_state, status, task);
    return sf::check_launch(TASK ? "kda chunk launch" : "kda_gated chunk launch", err, cap);
}

}  // namespace

// Chunked kernel for D = 128 with 16-byte-aligned q/k/v/g rows; returns SF_EINVAL (without
// launching) when the shape or alignment does not qualify.
int sf_kda_gated_chunk_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                              const void* initial_state, void* out, void* final_state, int64_t N, int64_t H, int64_t Dd, float scale,
                              int32_t dtype, cudaStream_t st, char* err, uint64_t cap) {
    return chunk_launch<false>(q, k, v, g, beta, cu_seqlens, initial_state, out, final_state, N, H, Dd, scale, TaskArgs{nullptr, nullptr, nullptr, 0.f},
                               dtype, st, err, cap);
}

// The task op (in-op norms and gates) on the chunked kernel; same qualification rules.
int sf_kda_task_chunk_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
                             const void* dt_bias, const void* initial_state, const void* cu_seqlens, const void* scale, void* out,
                             void* final_state, int64_t N, int64_t H, int64_t Dd, float lower_bound, int32_t dtype, cudaStream_t st,
                             char* err, uint64_t cap) {
    return chunk_launch<true>(q, k, v, g, beta, cu_seqlens, initial_state, out, final_state, N, H, Dd, 0.f,
                              TaskArgs{(const float*)a_log, (const float*)dt_bias, (const float*)scale, lower_bound}, dtype, st, err, cap);
}

int sf_kda_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream) {
    sm100::KernelStatus hs{0, 0};
    if (cudaMemcpyFromSymbolAsync(&hs, g_kda_status, sizeof(hs), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess) return SF_EDEVICE;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return SF_EDEVICE;
    if (hs.code) {
        const sm100::KernelStatus zero{0, 0};
        cudaMemcpyToSymbolAsync(g_kda_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream);
        cudaStreamSynchronize(stream);
    }
    *code = hs.code;
    *where = hs.where;
    return SF_OK;
}
