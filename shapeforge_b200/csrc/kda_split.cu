// Gated delta rule (the gated KDA workload) forward on sm_100a in two passes over a workspace,
// 32 tokens per chunk, D = 128.
//
// The chunk algebra is that of kda_c32.cu.  With b_t the cumulative log-decay from the chunk start
// (per channel), Kp_t = k_t e^{b_t}, Qp_t = q~_t e^{b_t} (q~ = q * scale), Kend_t = k_t e^{b_31 - b_t},
// A[t,i] = sum_c k_t k_i e^{b_t - b_i} (i < t), M[t,i] = sum_c q~_t k_i e^{b_t - b_i} (i <= t) and
// T = (I + diag(beta) A)^-1 diag(beta):
//   w = T V - (T Kp) S0^T     o = (M T) V + (Qp - M T Kp) S0^T     S <- S0 diag(e^{b_31}) + W^T Kend
// (the token recurrence of tasks/varlen_kda/reference.py:352-368 with the log-decay supplied,
// summed over a chunk).  Everything but the products with V and S depends on q, k, g and beta
// alone, so it is formed for all chunks at once, off the chain's critical path:
//
//  1. kda_slots_kernel: base[s] = number of 32-token chunks of the sequences before s.
//  2. kda_prep_kernel: one CTA per (sequence, head, chunk), three CTAs per SM.  It writes the
//     chunk's workspace slot, the exact shared-memory image the chain kernel's MMAs read:
//       B1  [-K2 ; Q2] fp32, MN-major (a 128-byte row of 32 tokens per channel, 32-byte
//           granules XOR-ed by channel & 3), -K2 then Q2 blocks of 128 rows        32768 B
//       KE  Kend 16-bit, MN-major, 2 blocks of 32 rows x 128 B            8192 B
//       TMB [T ; MT] 16-bit high | low, K-major rows of 128 B             8192 B
//       EL  e^{b_31} fp32 [128]                                             512 B
//  3. kda_chain_kernel: one CTA per (sequence, head) chain, the fp32 state [Dv, Dk] in TMEM.  A
//     producer warp streams the chain's slots (one bulk copy each) and V (cp.async, zero-filled past
//     the chain's end) through a 3-stage ring.  Two MMA warps issue, per chunk, the two K halves of
//     ACC += S [-K2 ; Q2]^T into the chunk's accumulator (already holding V^T [T ; MT]^T, so it ends
//     as w^T | o^T) and a second accumulator; the first then issues the next chunk's
//     V^T [T ; MT]^T into the other accumulator buffer while
//     eight state warps write W^T as 16-bit high | low parts and decay S, then S += W^T Kend; the
//     state warps store o after handing W^T over.
//
// Numerics match kda_c32.cu: the A and M factors e^{+-(b_t - r)} use the midpoint r of each channel's
// b range over the chunk, a chunk whose range exceeds 160 in some channel forms A and M pair by pair,
// per-token decays are floored at -200.  Every mbarrier wait is bounded and reports through
// sf_kernel_status; a workspace too small for the sequences (where = 95) or a sequence ending past the
// stated token count (where = 96) is reported there too, with no work done.
#include "kda_layout.cuh"
#include "sf_common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <atomic>
#include <type_traits>

__device__ sm100::KernelStatus g_kda_split_status;

namespace {

using kdal::chunk128;
using kdal::from16;
using kdal::kmaj32;
using kdal::mnmaj16;
using kdal::pack_hi_lo;
using kdal::to16;

constexpr int D = 128;
constexpr int C = 32;
constexpr float FACTOR_LIMIT = 80.f;
constexpr float DECAY_FLOOR = -200.f;

// Workspace slot image (bytes).
constexpr int SL_B1 = 0, SL_KE = 32768, SL_TMB = 40960, SL_EL = 49152, SLOT_BYTES = 49664;

__host__ __device__ inline int64_t header_bytes(int64_t nseq) { return ((4 * (nseq + 1) + 1023) / 1024) * 1024; }

__device__ __forceinline__ int chunks_of(const int32_t* cu, int s) {
    const int b = cu[s], e = cu[s + 1];
    return (b < 0 || e < 0 || e < b) ? 0 : (e - b + C - 1) / C;
}

__device__ __forceinline__ void report_bad_workspace(sm100::KernelStatus* st) {
    if (atomicCAS(&st->code, 0u, 2u) == 0u) st->where = 95u;
}

// ---------------------------------------------------------------------------------------------
// 1. chunk prefix over the sequences (one CTA of 1024 threads)
// ---------------------------------------------------------------------------------------------
// A sequence that ends past `total_tokens` (the rows the tensors were described with) makes the
// chunk total unreachable, so the later passes skip all work and report it (where = 96).
__global__ void __launch_bounds__(1024) kda_slots_kernel(const int32_t* __restrict__ cu, int nseq, int64_t total_tokens,
                                                          int32_t* __restrict__ base, sm100::KernelStatus* status) {
    __shared__ int part[32];
    __shared__ int bad;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    if (tid == 0) bad = 0;
    __syncthreads();
    const int per = (nseq + 1023) / 1024;
    const int s0 = min(nseq, tid * per), s1 = min(nseq, s0 + per);
    int sum = 0;
    for (int s = s0; s < s1; ++s) {
        sum += chunks_of(cu, s);
        if (chunks_of(cu, s) > 0 && (int64_t)cu[s + 1] > total_tokens) bad = 1;
    }
    int x = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) part[w] = x;
    __syncthreads();
    if (w == 0) {
        int y = part[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int z = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) y += z;
        }
        part[lane] = y;
    }
    __syncthreads();
    int excl = x - sum + (w > 0 ? part[w - 1] : 0);
    for (int s = s0; s < s1; ++s) {
        base[s] = excl;
        excl += chunks_of(cu, s);
    }
    if (tid == 1023) base[nseq] = bad ? 0x3fffffff : part[31];
    if (tid == 0 && bad && atomicCAS(&status->code, 0u, 2u) == 0u) status->where = 96u;
}

// ---------------------------------------------------------------------------------------------
// 2. prep: one chunk of one head per CTA
// ---------------------------------------------------------------------------------------------
constexpr int P_NT = 256;
struct PL {
    // q, k (2 x 64-channel boxes of 32 x 128 B each) and g (4 x 32-channel boxes) land here by TMA;
    // then [Kf ; Qf] fp32 MN-major (2 token blocks x 128 channel rows x 128 B); pairwise chunks: b
    // fp32 K-major 4 x (32 x 128 B); then the slot's KE | TMB | EL image (KE, then [T ; MT] 16-bit
    // high | low rows, then e^{b_31}), stored to the slot by one bulk copy.
    static constexpr int PA = 0;
    // Kn fp32 MN-major (128 channel rows x 128 B); then A, M, L^-1 / T, M T and P; finally (with
    // KP) the slot's B1 image, stored by one bulk copy.
    static constexpr int PB = 32768;
    static constexpr int KP = 51200;   // -Kp^T 16-bit K-major rows of 128 B: [channel][high 32 tokens | low 32 tokens]
    static constexpr int BS = 67584;   // beta [32] (0 past the chain's end)
    static constexpr int XTOT = BS + 128;
    static constexpr int XLAST = XTOT + 512;
    static constexpr int XLO = XLAST + 512;
    static constexpr int XHI = XLO + 1024;
    static constexpr int VOTE = XHI + 1024;  // 8 words
    static constexpr int INFO = VOTE + 32;   // valid, head, first token, token count
    static constexpr int BARS = INFO + 32;   // staged, p1, p4, TMEM base
    static constexpr int NRM = BARS + 32;    // task op: 1 / |q_t| [32], then 1 / |k_t| [32]
    static constexpr int DTB = NRM + 256;    // task op: dt_bias[h, 0..127]
    static constexpr int BYTES = DTB + 512;
};
constexpr int P_SQ = PL::PA, P_SK = PL::PA + 8192, P_SG = PL::PA + 16384;  // staged inputs inside PA
constexpr int TTS = 36;  // row stride of L^-1 / T (16-byte aligned rows for float4 reads)
constexpr int P_TA = PL::PB, P_TMM = P_TA + 4224, P_TT = P_TMM + 4224, P_TMT = P_TT + 4 * 32 * TTS, P_TP = P_TMT + 4224;
static_assert(P_TP + 16 * 17 * 4 <= PL::KP, "T matrices fit the Kn space");
static_assert(PL::PB % 1024 == 0 && PL::KP % 1024 == 0, "operand tiles are 1024-byte aligned");
constexpr uint32_t P_TM_D1 = 0, P_TM_D4 = 64, P_TMEM_COLS = 128;
constexpr uint32_t STAGED_BYTES = 32768, STAGED_BYTES_TASK = 24576;
constexpr int P_KE = PL::PA, P_TMB = PL::PA + 8192, P_EL = PL::PA + 16384, P_B1 = PL::PB;
static_assert(P_B1 + 32768 <= PL::BS, "B1 image fits PB and KP");

// Byte offset of fp32 element (MN index m, K index r) of an MN-major tf32 operand in the 32-byte
// granule swizzle (sm100::smem_desc_mn_b32): rows of 32 MN elements per K index, 4-row atoms of
// 512 B, 32-element MN blocks `blk` bytes apart.
__device__ __forceinline__ int mnmaj32(int m, int r, int blk) {
    return (m >> 5) * blk + r * 128 + ((((m & 31) >> 3) ^ (r & 3)) << 5) + ((m & 7) << 2);
}

// The task op's in-op transforms (tasks/varlen_kda/reference.py:323-374): q and k rows
// L2-normalised (rsqrt(sum x^2 + 1e-6), q times *scale), log-decay lower_bound *
// sigmoid(exp(A_log[h]) * (g + dt_bias[h, c])) from 16-bit g, beta = sigmoid(beta).
struct TaskGate {
    const float* a_log;    // [H]
    const float* dt_bias;  // [H * D]
    const float* scale;    // [1]
    float lower_bound;
};

// kind::tf32 instruction descriptor with both operands MN-major.
__host__ __device__ constexpr uint32_t idesc_tf32_mn(uint32_t m, uint32_t n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (1u << 15) | (1u << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// TASK: g and beta are 16-bit raw gates and the TaskGate transforms apply; otherwise g is the fp32
// log-decay, beta fp32 and q is multiplied by `scale`.
template <typename T, bool TASK>
__global__ void __launch_bounds__(P_NT, 3)
    kda_prep_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tg,
                    const T* __restrict__ q, const T* __restrict__ k, const void* __restrict__ beta, const int32_t* __restrict__ cu,
                    const int32_t* __restrict__ base, int nseq, int64_t max_slots, float scale, TaskGate task, int H,
                    uint8_t* __restrict__ slots, sm100::KernelStatus* status) {
    constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    int* info = reinterpret_cast<int*>(smem + PL::INFO);
    uint64_t* bar_ld = reinterpret_cast<uint64_t*>(smem + PL::BARS);
    uint64_t* bar_p1 = bar_ld + 1;
    uint64_t* bar_p4 = bar_ld + 2;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_ld + 3);

    const int p = threadIdx.x, lane = p & 31, pw = p >> 5;
    const int c = p & 127, half = p >> 7;
    const int64_t j = blockIdx.x;
    if (pw == 0) {
        // The slot's sequence: the last s with base[s] * H <= j, found by warp 0 in a 32-way search
        // (one round of loads for up to 32 sequences; base[0] = 0 keeps lane 0's probe true).
        const int64_t total = (int64_t)base[nseq] * H;
        int valid = 0, hh = 0, t0 = 0, nt = 0;
        if (total > max_slots) {
            if (j == 0 && lane == 0) report_bad_workspace(status);
        } else if (j < total) {
            int lo = 0, n = nseq;
            while (n > 1) {
                const int step = (n + 31) >> 5;
                const bool le = lane * step < n && (int64_t)base[lo + lane * step] * H <= j;
                const int last = 31 - __clz(__ballot_sync(0xffffffffu, le) | 1u);
                lo += last * step;
                n = min(step, n - last * step);
            }
            // base[lo], base[lo + 1], cu[lo], cu[lo + 1] in one round.
            const int x = lane < 2 ? base[lo + lane] : (lane < 4 ? cu[lo + lane - 2] : 0);
            const int b0 = __shfl_sync(0xffffffffu, x, 0), b1 = __shfl_sync(0xffffffffu, x, 1);
            const int c0 = __shfl_sync(0xffffffffu, x, 2), c1 = __shfl_sync(0xffffffffu, x, 3);
            const int64_t r = j - (int64_t)b0 * H;
            const int nch = b1 - b0;
            hh = (int)(r / nch);
            t0 = c0 + C * (int)(r % nch);
            nt = min(C, c1 - t0);
            valid = 1;
        }
        if (lane == 0 && valid) {
            // q, k, g of the chunk's 32 token rows (rows past the chain's end are read and then
            // ignored; rows past the tensor are zero-filled).
            sm100::mbar_init(bar_ld, 1);
            sm100::mbar_init(bar_p1, 1);
            sm100::mbar_init(bar_p4, 1);
            sm100::fence_mbar_init();
            sm100::mbar_arrive_expect_tx(bar_ld, TASK ? STAGED_BYTES_TASK : STAGED_BYTES);
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                sm100::tma_load_3d(smem + P_SQ + 4096 * b, &tq, bar_ld, 64 * b, hh, t0);
                sm100::tma_load_3d(smem + P_SK + 4096 * b, &tk, bar_ld, 64 * b, hh, t0);
            }
            // g: 16-bit boxes of 64 channels (task) or fp32 boxes of 32 channels.
#pragma unroll
            for (int b = 0; b < (TASK ? 2 : 4); ++b) sm100::tma_load_3d(smem + P_SG + 4096 * b, &tg, bar_ld, (TASK ? 64 : 32) * b, hh, t0);
        }
        if (lane == 0) {
            info[0] = valid;
            info[1] = hh;
            info[2] = t0;
            info[3] = nt;
            info[4] = 0;  // a bounded wait of thread 0 gave up
        }
    }
    __syncthreads();
    if (!info[0]) return;
    const int hh = info[1], t0 = info[2], nt = info[3];
    uint8_t* slot = slots + (size_t)j * SLOT_BYTES;
    if (pw == 0) {
        sm100::tmem_alloc(tslot, P_TMEM_COLS);
        sm100::tmem_relinquish();
    }
    float* bs = reinterpret_cast<float*>(smem + PL::BS);
    if (p < C) {
        float b = 0.f;
        if (p < nt) {
            if (TASK) b = 1.0f / (1.0f + __expf(-sf::Dt<T>::to_f(static_cast<const T*>(beta)[(size_t)(t0 + p) * H + hh])));
            else b = static_cast<const float*>(beta)[(size_t)(t0 + p) * H + hh];
        }
        bs[p] = b;
    }
    float* dtb = reinterpret_cast<float*>(smem + PL::DTB);
    if (TASK && p < D) dtb[p] = task.dt_bias[(size_t)hh * D + p];
    const float qscale = TASK ? *task.scale : scale;
    // Thread 0 alone waits for the staged inputs (and below, for each MMA); the other warps sleep
    // at the CTA barrier instead of polling.
    if (p == 0 && !sm100::mbar_wait(bar_ld, 0, status, 90)) info[4] = 1;
    __syncthreads();
    float* nrm = reinterpret_cast<float*>(smem + PL::NRM);
    if (TASK) {
        // 1 / |q_t| and 1 / |k_t|: thread -> token p / 8, channels 16 (p & 7) .. + 15 (two 16-byte
        // chunks of one 64-channel box row), the 8 threads of a token reduce by shuffles.  The same
        // thread turns its 16 gates into log-decays, written as fp32 into PB in the layout the fp32
        // g boxes of the gated workload have (box of 32 channels x 32 tokens, 128-byte swizzle),
        // where the factor pass reads them; PB is free until that pass writes Kn.
        const int tt = p >> 3, part = p & 7;
        const int roff = (part >> 2) * 4096 + tt * 128;
        const float ea = __expf(task.a_log[hh]);
        float sq = 0.f, sk = 0.f;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int co = ((2 * (part & 3) + u) ^ (tt & 7)) << 4;
            const uint4 qw = *reinterpret_cast<const uint4*>(smem + P_SQ + roff + co);
            const uint4 kw = *reinterpret_cast<const uint4*>(smem + P_SK + roff + co);
            const uint4 gw = *reinterpret_cast<const uint4*>(smem + P_SG + roff + co);
            const uint32_t qa[4] = {qw.x, qw.y, qw.z, qw.w}, ka[4] = {kw.x, kw.y, kw.z, kw.w}, ga[4] = {gw.x, gw.y, gw.z, gw.w};
            float ld[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float q0 = from16<T>((uint16_t)(qa[e] & 0xFFFFu)), q1 = from16<T>((uint16_t)(qa[e] >> 16));
                const float k0 = from16<T>((uint16_t)(ka[e] & 0xFFFFu)), k1 = from16<T>((uint16_t)(ka[e] >> 16));
                sq = fmaf(q0, q0, fmaf(q1, q1, sq));
                sk = fmaf(k0, k0, fmaf(k1, k1, sk));
                const int ch = 16 * part + 8 * u + 2 * e;
                const float g0 = from16<T>((uint16_t)(ga[e] & 0xFFFFu)), g1 = from16<T>((uint16_t)(ga[e] >> 16));
                ld[2 * e] = task.lower_bound * __fdividef(1.0f, 1.0f + __expf(-ea * (g0 + dtb[ch])));
                ld[2 * e + 1] = task.lower_bound * __fdividef(1.0f, 1.0f + __expf(-ea * (g1 + dtb[ch + 1])));
            }
            // Channels 16 part + 8 u .. + 7: two 16-byte chunks of box (part >> 1), row tt.
            uint8_t* gd = smem + PL::PB + (part >> 1) * 4096 + tt * 128;
#pragma unroll
            for (int v2 = 0; v2 < 2; ++v2) {
                const int chunk = 4 * (part & 1) + 2 * u + v2;
                *reinterpret_cast<float4*>(gd + ((chunk ^ (tt & 7)) << 4)) =
                    make_float4(ld[4 * v2], ld[4 * v2 + 1], ld[4 * v2 + 2], ld[4 * v2 + 3]);
            }
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
            sk += __shfl_xor_sync(0xffffffffu, sk, o);
        }
        if (part == 0) {
            nrm[tt] = rsqrtf(sq + 1e-6f);
            nrm[C + tt] = rsqrtf(sk + 1e-6f);
        }
        __syncthreads();
    }

    // ---- the thread's 16 tokens of channel c: log-decay, k, q~ (zero past the chain's end) ----
    // Channel c's element of token t = 16 * half + jj in a staged tile sits at the row base +
    // jj * 128 + (its 16-byte chunk XOR (jj & 7) * 16): t & 7 == jj & 7, so only the XOR varies.
    const int gch = ((c & 31) >> 2) << 4, hch = ((c & 63) >> 3) << 4;
    // fp32 log-decays: the staged g boxes, or (task op) the decays formed above in PB.
    const uint8_t* sg0 = smem + (TASK ? PL::PB : P_SG) + (c >> 5) * 4096 + half * 2048 + ((c & 3) << 2);
    const uint8_t* sk0 = smem + P_SK + (c >> 6) * 4096 + half * 2048 + ((c & 7) << 1);
    const uint8_t* sq0 = sk0 - P_SK + P_SQ;
    float bl[16], kv[16], qv[16];
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
        const bool live = 16 * half + jj < nt;
        const int rw = jj * 128;
        const float gl = *reinterpret_cast<const float*>(sg0 + rw + (gch ^ ((jj & 7) << 4)));
        float kx = from16<T>(*reinterpret_cast<const uint16_t*>(sk0 + rw + (hch ^ ((jj & 7) << 4))));
        float qx = from16<T>(*reinterpret_cast<const uint16_t*>(sq0 + rw + (hch ^ ((jj & 7) << 4)))) * qscale;
        if (TASK) {
            kx *= nrm[C + 16 * half + jj];
            qx *= nrm[16 * half + jj];
        }
        bl[jj] = live ? gl : 0.f;
        kv[jj] = live ? kx : 0.f;
        qv[jj] = live ? qx : 0.f;
    }
    sm100::tc_fence_before();
    __syncthreads();  // the staged inputs are consumed: PA is free for the factors
    sm100::tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t lane_q = (uint32_t)((pw & 3) * 32) << 16;

    float* xtot = reinterpret_cast<float*>(smem + PL::XTOT);
    float* xlast = reinterpret_cast<float*>(smem + PL::XLAST);
    float* xlo = reinterpret_cast<float*>(smem + PL::XLO);
    float* xhi = reinterpret_cast<float*>(smem + PL::XHI);
    uint32_t* vote = reinterpret_cast<uint32_t*>(smem + PL::VOTE);
    {
        float acc = 0.f;
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
            const float x = bl[jj] < DECAY_FLOOR ? DECAY_FLOOR : bl[jj];  // NaN passes through
            acc += x;
            bl[jj] = acc;
        }
        if (half == 0) xtot[c] = acc;
    }
    __syncthreads();
    if (half == 1) {
        const float off = xtot[c];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) bl[jj] += off;
    }
    {
        float lo = bl[0], hi = bl[0];
#pragma unroll
        for (int jj = 1; jj < 16; ++jj) {
            lo = fminf(lo, bl[jj]);
            hi = fmaxf(hi, bl[jj]);
        }
        xlo[half * 128 + c] = lo;
        xhi[half * 128 + c] = hi;
        if (half == 1) xlast[c] = bl[15];
    }
    __syncthreads();
    const float blo = fminf(xlo[c], xlo[128 + c]), bhi = fmaxf(xhi[c], xhi[128 + c]);
    const float blast = xlast[c];
    const float elast_c = kdal::fexp(blast);
    const float ref = 0.5f * (blo + bhi);
    const bool wide = !(0.5f * (bhi - blo) <= FACTOR_LIMIT);  // NaN counts as wide
    {
        const bool any = __any_sync(0xffffffffu, wide);
        if (lane == 0) vote[pw] = any ? 1u : 0u;
    }
    uint16_t kend16[16];  // the slot's Kend of the thread's tokens, written once PA is free
    {
        // Per group of 4 tokens: Kf, Qf (A rows) and Kn (B rows) of the A | M MMA as MN-major
        // fp32 vectors for a narrow channel; -Kp (high | low, a K-major row per channel) for the
        // K2 | M T Kp MMA; Kend into the slot; Qp seeds the M T Kp columns of that MMA's
        // accumulator (which then holds Q2), whose K2 columns start at zero.
        const float er = kdal::fexp(ref), elr = kdal::fexp(blast - ref);
        uint32_t qp[16], zero[16], kh[8], kl[8];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) zero[jj] = 0u;
        // The two paths are separate loops so that neither executes the other's exponentials.
        if (!wide) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float kf[4], qf[4], kn[4], kp[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int jj = 4 * u + e;
                    const float x = bl[jj] - ref;
                    const float ex = kdal::fexp(x), en = kdal::fexp(-x);
                    kf[e] = kv[jj] * ex;
                    qf[e] = qv[jj] * ex;
                    kn[e] = kv[jj] * en;
                    kp[e] = kf[e] * er;
                    qp[jj] = __float_as_uint(qf[e] * er);
                    kend16[jj] = to16<T>(kn[e] * elr);
                }
                const int m = 16 * half + 4 * u;
                *reinterpret_cast<float4*>(smem + PL::PA + mnmaj32(m, c, 16384)) = make_float4(kf[0], kf[1], kf[2], kf[3]);
                *reinterpret_cast<float4*>(smem + PL::PA + mnmaj32(C + m, c, 16384)) = make_float4(qf[0], qf[1], qf[2], qf[3]);
                *reinterpret_cast<float4*>(smem + PL::PB + mnmaj32(m, c, 16384)) = make_float4(kn[0], kn[1], kn[2], kn[3]);
                kh[2 * u] = kdal::pack_hi_lo2<T>(-kp[0], -kp[1], kl[2 * u]);
                kh[2 * u + 1] = kdal::pack_hi_lo2<T>(-kp[2], -kp[3], kl[2 * u + 1]);
            }
        } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float kp[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int jj = 4 * u + e;
                    const float e0 = kdal::fexp(bl[jj]);
                    kp[e] = kv[jj] * e0;
                    qp[jj] = __float_as_uint(qv[jj] * e0);
                    kend16[jj] = to16<T>(kv[jj] * kdal::fexp(blast - bl[jj]));
                }
                kh[2 * u] = kdal::pack_hi_lo2<T>(-kp[0], -kp[1], kl[2 * u]);
                kh[2 * u + 1] = kdal::pack_hi_lo2<T>(-kp[2], -kp[3], kl[2 * u + 1]);
            }
        }
        uint8_t* kprow = smem + PL::KP;
        *reinterpret_cast<uint4*>(kprow + chunk128(c, 2 * half)) = make_uint4(kh[0], kh[1], kh[2], kh[3]);
        *reinterpret_cast<uint4*>(kprow + chunk128(c, 2 * half + 1)) = make_uint4(kh[4], kh[5], kh[6], kh[7]);
        *reinterpret_cast<uint4*>(kprow + chunk128(c, 4 + 2 * half)) = make_uint4(kl[0], kl[1], kl[2], kl[3]);
        *reinterpret_cast<uint4*>(kprow + chunk128(c, 5 + 2 * half)) = make_uint4(kl[4], kl[5], kl[6], kl[7]);
        sm100::tmem_st_32x32b_x16(tmem + lane_q + P_TM_D4 + (uint32_t)(16 * half), zero);
        sm100::tmem_st_32x32b_x16(tmem + lane_q + P_TM_D4 + (uint32_t)(C + 16 * half), qp);
        sm100::tmem_st_wait();
    }
    sm100::tc_fence_before();
    sm100::fence_proxy_async_smem();
    __syncthreads();
    const bool exact = (vote[0] | vote[1] | vote[2] | vote[3] | vote[4] | vote[5] | vote[6] | vote[7]) != 0u;

    float* ta = reinterpret_cast<float*>(smem + P_TA);
    float* tmm = reinterpret_cast<float*>(smem + P_TMM);
    float* tt = reinterpret_cast<float*>(smem + P_TT);
    float* tmt = reinterpret_cast<float*>(smem + P_TMT);
    float* tp = reinterpret_cast<float*>(smem + P_TP);
    if (!exact) {
        // ---- A | M = [Kf ; Qf] . Kn^T: M = 64, N = 32, K = 128 (tf32, both operands MN-major) ----
        if (p == 0) {
            sm100::tc_fence_after();
            constexpr uint32_t idesc = idesc_tf32_mn(64, 32);
            const uint64_t ad0 = sm100::smem_desc_mn_b32(sm100::smem_u32(smem + PL::PA), 16384, 512);
            const uint64_t bd0 = sm100::smem_desc_mn_b32(sm100::smem_u32(smem + PL::PB), 16384, 512);
#pragma unroll
            for (int kk = 0; kk < D / 8; ++kk)
                sm100::mma_tf32(tmem + P_TM_D1, ad0 + (uint64_t)((kk * 1024) >> 4), bd0 + (uint64_t)((kk * 1024) >> 4), idesc,
                                kk > 0 ? 1u : 0u);
            sm100::mma_commit(bar_p1);
            if (!sm100::mbar_wait(bar_p1, 0, status, 91)) info[4] = 1;
            sm100::tc_fence_before();
        }
        __syncthreads();
        sm100::tc_fence_after();
        {
            // M=64 layout: rows 16*i + r sit in TMEM lane 32*i + r (r < 16).  Quadrants 0/1: A rows
            // 0-15 / 16-31; quadrants 2/3: M rows 0-15 / 16-31.  Warps 0-3 take columns 0-15,
            // warps 4-7 columns 16-31.  A and M overwrite Kn, which the MMA has consumed.
            uint32_t r[16];
            sm100::tmem_ld_32x32b_x16(tmem + lane_q + P_TM_D1 + (uint32_t)((pw >> 2) * 16), r);
            sm100::tmem_ld_wait();
            if (lane < 16) {
                const int qd = pw & 3;
                const int t = (qd & 1) * 16 + lane;
                float* dst = qd < 2 ? ta : tmm;
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) {
                    const int i = (pw >> 2) * 16 + jj;
                    const bool keep = qd < 2 ? (i < t) : (i <= t);
                    dst[t * 33 + i] = keep ? __uint_as_float(r[jj]) : 0.f;
                }
            }
        }
    } else {
        // ---- pairwise A and M (any decay): b into PA, thread -> row t, columns i0 + 8u ----
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) *reinterpret_cast<float*>(smem + PL::PA + kmaj32(16 * half + jj, c, 4096)) = bl[jj];
        __syncthreads();
        const int t = p >> 3, i0 = p & 7;
        float a[4] = {0.f, 0.f, 0.f, 0.f}, m[4] = {0.f, 0.f, 0.f, 0.f};
        if (t < nt) {
            const size_t rt = ((size_t)(t0 + t) * H + hh) * D;
#pragma unroll 2
            for (int cc = 0; cc < D; ++cc) {
                const int col = (cc + 4 * i0) & (D - 1);
                const float bt = *reinterpret_cast<const float*>(smem + PL::PA + kmaj32(t, col, 4096));
                const float kt = sf::Dt<T>::to_f(k[rt + col]);
                const float qt = sf::Dt<T>::to_f(q[rt + col]);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int i = i0 + 8 * u;
                    if (i <= t) {
                        const float bi = *reinterpret_cast<const float*>(smem + PL::PA + kmaj32(i, col, 4096));
                        const float ki = sf::Dt<T>::to_f(k[((size_t)(t0 + i) * H + hh) * D + col]) * __expf(bt - bi);
                        a[u] = fmaf(kt, ki, a[u]);
                        m[u] = fmaf(qt, ki, m[u]);
                    }
                }
            }
        }
        // The raw q, k rows read above take the task op's norms here (and q its scale).
        const float nkt = TASK ? nrm[C + t] : 1.f, nqt = TASK ? nrm[t] * qscale : qscale;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = i0 + 8 * u;
            const bool live = t < nt && i < nt;
            const float nki = TASK ? nrm[C + i] : 1.f;
            ta[t * 33 + i] = (live && i < t) ? a[u] * nkt * nki : 0.f;
            tmm[t * 33 + i] = (live && i <= t) ? m[u] * nqt * nki : 0.f;
        }
    }
    __syncthreads();  // A and M are written; PA (factors or b) is consumed
    {
        // Kend into the KE image (MN-major 16-bit: token rows of 128 B per 64-channel block).
        uint8_t* ke0 = smem + P_KE + (c >> 6) * 4096 + half * 2048 + ((c & 7) << 1);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) *reinterpret_cast<uint16_t*>(ke0 + jj * 128 + (hch ^ ((jj & 7) << 4))) = kend16[jj];
        if (half == 0) reinterpret_cast<float*>(smem + P_EL)[c] = elast_c;
    }
    // ---- T = (I + diag(beta) A)^-1 diag(beta) in 16 x 16 blocks ----
    if (p < 32) {
        const int bb = p >> 4, jc = p & 15, o = 16 * bb;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < r; ++i) acc = fmaf(ta[(o + r) * 33 + o + i], x[i], acc);
            x[r] = (r == jc ? 1.f : 0.f) - bs[o + r] * acc;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) tt[(o + r) * TTS + o + jc] = x[r];
    }
    __syncthreads();
    {
        // P = diag(beta_2) A21 L11^-1, then L21^-1 = -L22^-1 P; the upper-right block is 0.
        const int r = p >> 4, jc = p & 15;
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) acc = fmaf(ta[(16 + r) * 33 + i], tt[i * TTS + jc], acc);
        tp[r * 17 + jc] = bs[16 + r] * acc;
        tt[r * TTS + 16 + jc] = 0.f;
    }
    __syncthreads();
    {
        const int r = p >> 4, jc = p & 15;
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) acc = fmaf(tt[(16 + r) * TTS + 16 + i], tp[i * 17 + jc], acc);
        tt[(16 + r) * TTS + jc] = -acc;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int e = p + P_NT * u, r = e >> 5, jc = e & 31;
        tt[r * TTS + jc] *= bs[jc];
    }
    __syncthreads();
    {
        // M T: thread -> row r, columns 4 j0 .. 4 j0 + 3 (M and T hold zeros above their diagonals).
        const int r = p >> 3, j0 = p & 7;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < C; ++i) {
            const float mri = tmm[r * 33 + i];
            const float4 tv = *reinterpret_cast<const float4*>(tt + i * TTS + 4 * j0);
            acc[0] = fmaf(mri, tv.x, acc[0]);
            acc[1] = fmaf(mri, tv.y, acc[1]);
            acc[2] = fmaf(mri, tv.z, acc[2]);
            acc[3] = fmaf(mri, tv.w, acc[3]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) tmt[r * 33 + 4 * j0 + u] = acc[u];
    }
    __syncthreads();
    {
        // [T ; MT] as 16-bit high | low rows (thread -> row n, 8 columns) into the TMB image: the
        // next MMA's B operand and the slot's copy for the chain.
        const int n = p >> 2, i0 = (p & 3) * 8;
        const float* src = n < C ? tt + n * TTS : tmt + (n - C) * 33;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) hi[u] = pack_hi_lo<T>(src[i0 + 2 * u], src[i0 + 2 * u + 1], lo[u]);
        *reinterpret_cast<uint4*>(smem + P_TMB + chunk128(n, i0 >> 3)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(smem + P_TMB + chunk128(n, 4 + (i0 >> 3))) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    sm100::fence_proxy_async_smem();
    __syncthreads();

    // ---- [-K2 | Q2] = [0 | Qp] + (-Kp)^T . [T ; MT]^T: M = 128 (channels), N = 64, K = 32, bf16 x3, both K-major ----
    if (p == 0) {
        // The KE | TMB | EL part of the slot is final: its bulk store overlaps the MMA below.
        sm100::bulk_store(slot + SL_KE, sm100::smem_u32(smem + P_KE), SLOT_BYTES - SL_KE);
        sm100::bulk_commit();
        sm100::tc_fence_after();
        constexpr uint32_t idesc = sm100::idesc_f16(128, 64, BF16);
        const uint64_t ad0 = sm100::smem_desc_k_sw128(sm100::smem_u32(smem + PL::KP));
        const uint64_t bd0 = sm100::smem_desc_k_sw128(sm100::smem_u32(smem + P_TMB));
#pragma unroll
        for (int part = 0; part < 3; ++part) {
            const uint32_t a_part = part == 2 ? 64u : 0u;  // -Kp high, high, low
            const uint32_t b_part = part == 1 ? 64u : 0u;  // [T ; MT] high, low, high
#pragma unroll
            for (int kk = 0; kk < 2; ++kk)
                sm100::mma_f16(tmem + P_TM_D4, ad0 + (uint64_t)((a_part + kk * 32) >> 4), bd0 + (uint64_t)((b_part + kk * 32) >> 4),
                               idesc, 1u);
        }
        sm100::mma_commit(bar_p4);
        if (!sm100::mbar_wait(bar_p4, 0, status, 92)) info[4] = 1;
        sm100::tc_fence_before();
    }
    __syncthreads();
    sm100::tc_fence_after();
    if (!info[4]) {
        uint32_t k2r[16], q2r[16];
        sm100::tmem_ld_32x32b_x16(tmem + lane_q + P_TM_D4 + (uint32_t)(16 * half), k2r);
        sm100::tmem_ld_32x32b_x16(tmem + lane_q + P_TM_D4 + (uint32_t)(C + 16 * half), q2r);
        sm100::tmem_ld_wait();
        // B1 image, MN-major (row = channel, 32 tokens per 128-byte row, 32-byte granules XOR-ed
        // by c & 3): the thread's 16 tokens are two granules of -K2 and two of Q2.  PB and KP are
        // free: the K2 | M T Kp MMA has completed.
        uint8_t* b1 = smem + P_B1 + c * 128;
#pragma unroll
        for (int gq = 0; gq < 2; ++gq) {
            const int go = ((2 * half + gq) ^ (c & 3)) << 5;
            *reinterpret_cast<uint4*>(b1 + go) = make_uint4(k2r[8 * gq], k2r[8 * gq + 1], k2r[8 * gq + 2], k2r[8 * gq + 3]);
            *reinterpret_cast<uint4*>(b1 + go + 16) = make_uint4(k2r[8 * gq + 4], k2r[8 * gq + 5], k2r[8 * gq + 6], k2r[8 * gq + 7]);
            *reinterpret_cast<uint4*>(b1 + 16384 + go) = make_uint4(q2r[8 * gq], q2r[8 * gq + 1], q2r[8 * gq + 2], q2r[8 * gq + 3]);
            *reinterpret_cast<uint4*>(b1 + 16384 + go + 16) =
                make_uint4(q2r[8 * gq + 4], q2r[8 * gq + 5], q2r[8 * gq + 6], q2r[8 * gq + 7]);
        }
    }
    // B1 (32 KB) by a second bulk copy; the CTA leaves once both copies have read shared memory
    // (the chain kernel is a later launch on the same stream).
    sm100::fence_proxy_async_smem();
    __syncthreads();
    if (p == 0) {
        sm100::bulk_store(slot + SL_B1, sm100::smem_u32(smem + P_B1), 32768);
        sm100::bulk_commit();
        sm100::bulk_wait_read();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (pw == 0) sm100::tmem_dealloc(tmem, P_TMEM_COLS);
}

// ---------------------------------------------------------------------------------------------
// 3. chain: one (sequence, head) per CTA
// ---------------------------------------------------------------------------------------------
constexpr int K_NT = 352;  // warps 0-7 state, warp 8 producer, warps 9 and 10 MMA issue
constexpr int NSTAGE = 3;
constexpr int STAGE_V = 50176;  // V of the chunk, 16-bit MN-major 2 x (32 x 128 B), after the slot image
constexpr int STAGE_BYTES = STAGE_V + 8192;
struct KL {
    static constexpr int WT = NSTAGE * STAGE_BYTES;  // [W_hi | W_lo]^T K-major rows of 128 B, 128 rows
    static constexpr int OS = WT + 16384;            // o of a chunk [32 t][128 v] 16-bit
    static constexpr int BARS = OS + 8192;
    static constexpr int BYTES = BARS + 128;
};
static_assert(STAGE_V % 1024 == 0 && STAGE_BYTES % 1024 == 0 && KL::WT % 1024 == 0, "operand tiles are 1024-byte aligned");
static_assert(SLOT_BYTES <= STAGE_V, "slot image fits before V");

struct __align__(8) ChainBars {
    uint64_t full[NSTAGE];   // slot (transaction bytes) and V (32 cp.async arrivals) of a chunk landed
    uint64_t empty[NSTAGE];  // the chunk's state update done (commit): the stage may be refilled
    uint64_t m1;             // w | o accumulator ready (a commit from each MMA-issuing warp)
    uint64_t wready;         // W^T written and S decayed (one arrival per state warp)
    uint64_t oread[2];       // o read out of accumulator buffer b (one arrival per o warp); one
                             // barrier per buffer, so a wait can never alias a later chunk's phase
    uint64_t sinit;          // initial state in TMEM (one arrival per state warp)
    uint32_t tmem_base;
};
// TMEM: the state, then the w | o accumulator in two buffers (chunk parity), so the o warps can read
// a chunk's o after the hand-off while the next chunk's MMAs fill the other buffer; the S-product's
// second K half goes to a second accumulator pair (its own issuing warp), summed in the epilogue.
constexpr uint32_t TM_S = 0, TM_ACC = 128, TM_ACC2 = 256, K_TMEM_COLS = 512;

// r[j] *= e[j] for 32 state columns (e: 16-byte aligned shared memory).
__device__ __forceinline__ void decay32(uint32_t (&r)[32], const float* e) {
    const float4* e4 = reinterpret_cast<const float4*>(e);
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
        const float4 x = e4[j4];
        r[4 * j4] = __float_as_uint(__uint_as_float(r[4 * j4]) * x.x);
        r[4 * j4 + 1] = __float_as_uint(__uint_as_float(r[4 * j4 + 1]) * x.y);
        r[4 * j4 + 2] = __float_as_uint(__uint_as_float(r[4 * j4 + 2]) * x.z);
        r[4 * j4 + 3] = __float_as_uint(__uint_as_float(r[4 * j4 + 3]) * x.w);
    }
}

template <typename T>
__global__ void __launch_bounds__(K_NT, 1)
    kda_chain_kernel(const T* __restrict__ v, const int32_t* __restrict__ cu, const int32_t* __restrict__ base, int nseq,
                     int64_t max_slots, const float* __restrict__ state0, int H, const uint8_t* __restrict__ slots, T* __restrict__ out,
                     float* __restrict__ final_state, sm100::KernelStatus* status) {
    constexpr bool BF16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    ChainBars* bars = reinterpret_cast<ChainBars*>(smem + KL::BARS);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int s = blockIdx.x / H, h = blockIdx.x % H;
    const int begin = cu[s], end = cu[s + 1];
    if (begin < 0 || end < 0 || end < begin) return;  // sentinel: not part of this batch
    if ((int64_t)base[nseq] * H > max_slots) {
        if (tid == 0) report_bad_workspace(status);
        return;
    }
    const int ntok = end - begin;
    const int nch = (ntok + C - 1) / C;
    const int64_t slot0 = (int64_t)base[s] * H + (int64_t)h * nch;

    if (tid == 0) {
        for (int i = 0; i < NSTAGE; ++i) {
            sm100::mbar_init(&bars->full[i], 33);
            sm100::mbar_init(&bars->empty[i], 1);
        }
        sm100::mbar_init(&bars->m1, 2);
        sm100::mbar_init(&bars->wready, 8);
        sm100::mbar_init(&bars->oread[0], 4);
        sm100::mbar_init(&bars->oread[1], 4);
        sm100::mbar_init(&bars->sinit, 8);
        sm100::fence_mbar_init();
    }
    if (warp == 0) {
        sm100::tmem_alloc(&bars->tmem_base, K_TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem = bars->tmem_base;
    bool ok = true;

    if (warp == 8) {
        // ======================= producer =======================
        for (int ci = 0; ci < nch; ++ci) {
            const int st = ci % NSTAGE, n = ci / NSTAGE;
            if (ci >= NSTAGE && !sm100::mbar_wait(&bars->empty[st], (n - 1) & 1, status, 100)) ok = false;
            uint8_t* stg = smem + st * STAGE_BYTES;
            if (lane == 0) {
                sm100::mbar_arrive_expect_tx(&bars->full[st], SLOT_BYTES);
                sm100::bulk_load(sm100::smem_u32(stg), slots + (size_t)(slot0 + ci) * SLOT_BYTES, SLOT_BYTES, &bars->full[st]);
            }
            const int t0 = begin + ci * C, nt = min(C, end - t0);
            const uint32_t vb = sm100::smem_u32(stg + STAGE_V);
#pragma unroll
            for (int m = 0; m < 16; ++m) {
                const int id = lane + 32 * m;  // 512 chunks of 16 B: (t, j16)
                const int t = id >> 4, j16 = id & 15;
                const bool live = t < nt;
                const size_t row = ((size_t)(t0 + (live ? t : 0)) * H + h) * D + 8 * j16;
                sm100::cp_async_16(vb + (j16 >> 3) * 4096 + chunk128(t, j16), v + row, live ? 16u : 0u);
            }
            sm100::cp_async_mbar_arrive(&bars->full[st]);
        }
        // The copies of the last chunks have landed before the CTA can exit.
        for (int ci = max(0, nch - NSTAGE); ci < nch; ++ci)
            if (!sm100::mbar_wait(&bars->full[ci % NSTAGE], (ci / NSTAGE) & 1, status, 104)) ok = false;
    } else if (warp == 9) {
        // ======================= MMA issue (lane 0) =======================
        // Per chunk: the first K half of S [-K2 ; Q2]^T into the chunk's accumulator (which already
        // holds V^T [T ; MT]^T; warp 10 issues the second half into the second accumulator at the
        // same time), then -- while the state warps run the chunk's epilogue -- the next chunk's
        // V^T [T ; MT]^T into the other accumulator buffer, then S += W^T Kend once the epilogue
        // hands W^T over.  The tensor pipe executes one thread's MMAs in issue order; MMA issue is
        // per issuing thread, so the two halves take half the time of one thread's 16 MMAs.
        if (lane == 0 && nch > 0) {
            constexpr uint32_t idv = sm100::idesc_f16_major(128, 64, BF16, true, false);
            constexpr uint32_t idt = sm100::idesc_tf32(128, 64) | (1u << 16);  // B MN-major
            constexpr uint32_t idu = sm100::idesc_f16_bmn(128, D, BF16);
            auto issue_v = [&](int ci) {
                uint8_t* stg = smem + (ci % NSTAGE) * STAGE_BYTES;
                const uint32_t acc_t = tmem + TM_ACC + (uint32_t)(64 * (ci & 1));
                const uint64_t vd0 = sm100::smem_desc_mn_sw128(sm100::smem_u32(stg + STAGE_V), 4096, 1024);
                const uint64_t td0 = sm100::smem_desc_k_sw128(sm100::smem_u32(stg + SL_TMB));
#pragma unroll
                for (int part = 0; part < 2; ++part) {
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk)
                        sm100::mma_f16(acc_t, vd0 + (uint64_t)((kk * 2048) >> 4), td0 + (uint64_t)((part * 64 + kk * 32) >> 4), idv,
                                       (part | kk) != 0 ? 1u : 0u);
                }
            };
            if (!sm100::mbar_wait_spin(&bars->full[0], 0, status, 101)) ok = false;
            sm100::tc_fence_after();
            if (ok) issue_v(0);
            if (!sm100::mbar_wait_spin(&bars->sinit, 0, status, 107)) ok = false;
            sm100::tc_fence_after();
            for (int ci = 0; ci < nch; ++ci) {
                const int st = ci % NSTAGE;
                uint8_t* stg = smem + st * STAGE_BYTES;
                if (ok) {
                    const uint32_t acc_t = tmem + TM_ACC + (uint32_t)(64 * (ci & 1));
                    const uint64_t b1d = sm100::smem_desc_mn_b32(sm100::smem_u32(stg + SL_B1), 16384, 512);
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk)
                        sm100::mma_tf32_ta(acc_t, tmem + TM_S + (uint32_t)(kk * 8), b1d + (uint64_t)((kk * 1024) >> 4), idt, 1u);
                }
                sm100::mma_commit(&bars->m1);
                if (ci + 1 < nch) {
                    const int cn = ci + 1;
                    if (!sm100::mbar_wait_spin(&bars->full[cn % NSTAGE], (cn / NSTAGE) & 1, status, 101)) ok = false;
                    // The buffer's previous chunk (cn - 2, its ((cn - 2) / 2)-th use) has had its o read out.
                    if (cn >= 2 && !sm100::mbar_wait_spin(&bars->oread[cn & 1], ((cn - 2) >> 1) & 1, status, 108)) ok = false;
                    sm100::tc_fence_after();
                    if (ok) issue_v(cn);
                }
                if (!sm100::mbar_wait_spin(&bars->wready, ci & 1, status, 103)) ok = false;
                sm100::tc_fence_after();
                if (ok) {
                    const uint64_t wd0 = sm100::smem_desc_k_sw128(sm100::smem_u32(smem + KL::WT));
                    const uint64_t kd0 = sm100::smem_desc_mn_sw128(sm100::smem_u32(stg + SL_KE), 4096, 1024);
#pragma unroll
                    for (int part = 0; part < 2; ++part) {
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk)
                            sm100::mma_f16(tmem + TM_S, wd0 + (uint64_t)((part * 64 + kk * 32) >> 4), kd0 + (uint64_t)((kk * 2048) >> 4), idu,
                                           1u);
                    }
                }
                sm100::mma_commit(&bars->empty[st]);
            }
        }
        __syncwarp();
    } else if (warp == 10) {
        // ======================= second MMA issuer (lane 0) =======================
        // The second K half of the chunk's S-product into its second accumulator (initialised by
        // the first MMA).  Another thread's MMAs are not ordered with this one's, so it waits for
        // the state it reads: the initial state, then each chunk's update completed (empty), and
        // for the buffer's previous o having been read out.
        if (lane == 0 && nch > 0) {
            constexpr uint32_t idt = sm100::idesc_tf32(128, 64) | (1u << 16);  // B MN-major
            if (!sm100::mbar_wait_spin(&bars->sinit, 0, status, 109)) ok = false;
            for (int ci = 0; ci < nch; ++ci) {
                const int st = ci % NSTAGE;
                if (ci > 0 && !sm100::mbar_wait_spin(&bars->empty[(ci - 1) % NSTAGE], ((ci - 1) / NSTAGE) & 1, status, 110)) ok = false;
                if (!sm100::mbar_wait_spin(&bars->full[st], (ci / NSTAGE) & 1, status, 111)) ok = false;
                if (ci >= 2 && !sm100::mbar_wait_spin(&bars->oread[ci & 1], ((ci - 2) >> 1) & 1, status, 112)) ok = false;
                sm100::tc_fence_after();
                if (ok) {
                    const uint32_t acc2 = tmem + TM_ACC2 + (uint32_t)(64 * (ci & 1));
                    const uint64_t b1d = sm100::smem_desc_mn_b32(sm100::smem_u32(smem + st * STAGE_BYTES + SL_B1), 16384, 512);
#pragma unroll
                    for (int kk = D / 16; kk < D / 8; ++kk)
                        sm100::mma_tf32_ta(acc2, tmem + TM_S + (uint32_t)(kk * 8), b1d + (uint64_t)((kk * 1024) >> 4), idt,
                                           kk > D / 16 ? 1u : 0u);
                }
                sm100::mma_commit(&bars->m1);
            }
        }
        __syncwarp();
    } else {
        // ======================= state: value row v, S columns [64 * role, 64 * role + 64) =======================
        const int qd = warp & 3, role = warp >> 2;  // role 0: w, role 1: o
        const int vr = qd * 32 + lane;
        const uint32_t lane_q = (uint32_t)(qd * 32) << 16;
        const size_t srow = (((size_t)s * H + h) * D + vr) * D;
        const int cb0 = 64 * role;
#pragma unroll 1
        for (int cb = 0; cb < 2; ++cb) {
            uint32_t r[32];
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) r[jj] = __float_as_uint(state0 ? state0[srow + cb0 + 32 * cb + jj] : 0.f);
            sm100::tmem_st_32x32b_x32(tmem + lane_q + TM_S + (uint32_t)(cb0 + 32 * cb), r);
        }
        sm100::tmem_st_wait();
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&bars->sinit);
        for (int ci = 0; ci < nch; ++ci) {
            const int st = ci % NSTAGE, n = ci / NSTAGE;
            const int t0 = begin + ci * C, nt = min(C, end - t0);
            uint8_t* stg = smem + st * STAGE_BYTES;
            const uint32_t acc_t = tmem + TM_ACC + (uint32_t)(64 * (ci & 1));
            const uint32_t acc2_t = tmem + TM_ACC2 + (uint32_t)(64 * (ci & 1));
            // Thread 0 waits for the chunk's slot (its e^{b_31}) and accumulator; the other seven
            // warps sleep at the barrier instead of polling.
            if (tid == 0) {
                if (!sm100::mbar_wait(&bars->full[st], n & 1, status, 105)) ok = false;
                if (!sm100::mbar_wait_spin(&bars->m1, ci & 1, status, 102)) ok = false;
                sm100::tc_fence_before();
            }
            sm100::named_barrier_sync(1, 256);
            sm100::tc_fence_after();
            // Epilogue, split evenly: warp group r (r = 0, 1) packs W^T's tokens 16r .. 16r+15 (high |
            // low) and decays S columns 64r .. 64r+63; group 1 also takes o, which it stores after
            // the hand-off, off the critical path.
            const float* el = reinterpret_cast<const float*>(stg + SL_EL) + 64 * role;
            const uint32_t scol = tmem + lane_q + TM_S + (uint32_t)(64 * role);
            uint32_t wv[16], wv2[16], r0[32], r1[32];
            sm100::tmem_ld_32x32b_x16(acc_t + lane_q + (uint32_t)(16 * role), wv);
            sm100::tmem_ld_32x32b_x16(acc2_t + lane_q + (uint32_t)(16 * role), wv2);
            sm100::tmem_ld_32x32b_x32(scol, r0);
            sm100::tmem_ld_32x32b_x32(scol + 32u, r1);
            sm100::tmem_ld_wait();
#pragma unroll
            for (int u = 0; u < 16; ++u) wv[u] = __float_as_uint(__uint_as_float(wv[u]) + __uint_as_float(wv2[u]));
            {
                uint32_t hi[8], lo[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) hi[u] = kdal::pack_hi_lo2<T>(__uint_as_float(wv[2 * u]), __uint_as_float(wv[2 * u + 1]), lo[u]);
                uint8_t* row = smem + KL::WT;
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    *reinterpret_cast<uint4*>(row + chunk128(vr, 2 * role + jj)) =
                        make_uint4(hi[4 * jj], hi[4 * jj + 1], hi[4 * jj + 2], hi[4 * jj + 3]);
                    *reinterpret_cast<uint4*>(row + chunk128(vr, 4 + 2 * role + jj)) =
                        make_uint4(lo[4 * jj], lo[4 * jj + 1], lo[4 * jj + 2], lo[4 * jj + 3]);
                }
            }
            decay32(r0, el);
            decay32(r1, el + 32);
            sm100::tmem_st_32x32b_x32(scol, r0);
            sm100::tmem_st_32x32b_x32(scol + 32u, r1);
            sm100::tmem_st_wait();
            sm100::fence_proxy_async_smem();
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(&bars->wready);  // W^T written and S decayed (this warp's rows)
            if (role == 1) {
                // o^T row v (this chunk's accumulator buffer, which the next chunk's MMAs do not
                // touch) -> o [t][v] in shared memory, then whole 256-byte token rows to global
                // with 16-byte stores (rows past the chain's end are not stored).
                uint32_t a[32], a2[32];
                sm100::tmem_ld_32x32b_x32(acc_t + lane_q + (uint32_t)C, a);
                sm100::tmem_ld_32x32b_x32(acc2_t + lane_q + (uint32_t)C, a2);
                sm100::tmem_ld_wait();
#pragma unroll
                for (int t = 0; t < C; ++t) a[t] = __float_as_uint(__uint_as_float(a[t]) + __uint_as_float(a2[t]));
                sm100::tc_fence_before();
                __syncwarp();
                if (lane == 0) sm100::mbar_arrive(&bars->oread[ci & 1]);  // the buffer may take chunk ci + 2
                uint16_t* os = reinterpret_cast<uint16_t*>(smem + KL::OS);
#pragma unroll
                for (int t = 0; t < C; ++t) os[t * D + vr] = to16<T>(__uint_as_float(a[t]));
                sm100::named_barrier_sync(2, 128);
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const int id = vr + 128 * m, t = id >> 4, jj = id & 15;
                    if (t < nt)
                        *reinterpret_cast<uint4*>(out + ((size_t)(t0 + t) * H + h) * D + 8 * jj) =
                            *reinterpret_cast<const uint4*>(smem + KL::OS + t * 256 + 16 * jj);
                }
                sm100::named_barrier_sync(2, 128);
            }
        }
        // ---- final state ----
        if (tid == 0 && nch > 0 && !sm100::mbar_wait(&bars->empty[(nch - 1) % NSTAGE], ((nch - 1) / NSTAGE) & 1, status, 106))
            ok = false;
        sm100::tc_fence_before();
        sm100::named_barrier_sync(1, 256);
        sm100::tc_fence_after();
        ok = ok && *reinterpret_cast<volatile unsigned int*>(&status->code) == 0;
        if (ok) {
#pragma unroll 1
            for (int cb = 0; cb < 2; ++cb) {
                const int col = cb0 + 32 * cb;
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(tmem + lane_q + TM_S + (uint32_t)col, r);
                sm100::tmem_ld_wait();
                float4* dst = reinterpret_cast<float4*>(final_state + srow + col);
#pragma unroll
                for (int jj = 0; jj < 8; ++jj)
                    dst[jj] = make_float4(__uint_as_float(r[4 * jj]), __uint_as_float(r[4 * jj + 1]), __uint_as_float(r[4 * jj + 2]),
                                          __uint_as_float(r[4 * jj + 3]));
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 0) sm100::tmem_dealloc(tmem, K_TMEM_COLS);
}

sm100::KernelStatus* status_ptr() {
    sm100::KernelStatus* p = nullptr;
    if (cudaGetSymbolAddress((void**)&p, g_kda_split_status) != cudaSuccess) return nullptr;
    return p;
}

constexpr int PREP_SMEM = PL::BYTES + 1024;
constexpr int CHAIN_SMEM = KL::BYTES + 1024;

int64_t slot_bound(int64_t total_tokens, int64_t nseq, int64_t H) { return ((total_tokens + (C - 1) * nseq) / C) * H; }

}  // namespace

// Workspace bytes of the two-pass kernels for `total_tokens` tokens in `nseq` sequences of H heads
// (0 when the shape does not qualify: D != 128).
uint64_t sf_kda_gated_split_workspace(int64_t total_tokens, int64_t nseq, int64_t H, int64_t Dd) {
    if (Dd != D || nseq <= 0 || H <= 0 || total_tokens < 0) return 0;
    return (uint64_t)(header_bytes(nseq) + slot_bound(total_tokens, nseq, H) * SLOT_BYTES);
}

namespace {

template <bool TASK>
int split_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                 const void* initial_state, void* out, void* final_state, int64_t N, int64_t total_tokens, int64_t H, int64_t Dd,
                 float scale, TaskGate task, int32_t dtype, void* workspace, uint64_t workspace_bytes, cudaStream_t st, char* err,
                 uint64_t cap) {
    if (Dd != D || !sf::aligned16(q) || !sf::aligned16(k) || !sf::aligned16(v) || !sf::aligned16(g) || !sf::aligned16(out) ||
        !sf::aligned16(final_state) || (initial_state && !sf::aligned16(initial_state)))
        return sf::fail(SF_EINVAL, err, cap, "kda: the two-pass kernels need D = 128 and 16-byte-aligned tensors");
    if (N * H > 0x7fffffffLL || N >= 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "kda: too many chains");
    if (total_tokens < 0) return sf::fail(SF_EINVAL, err, cap, "kda: negative token count");
    const uint64_t need = sf_kda_gated_split_workspace(total_tokens, N, H, Dd);
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return sf::fail(SF_EINVAL, err, cap, "kda: the two-pass kernels need a 256-byte-aligned workspace of %llu bytes",
                        (unsigned long long)need);
    const int64_t nslots = slot_bound(total_tokens, N, H);
    if (nslots > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "kda: too many chunks");
    sm100::KernelStatus* status = status_ptr();
    if (!status) return sf::fail(SF_EDEVICE, err, cap, "kda: cannot resolve the status word");
    static std::atomic<uint64_t> attr_done{0};
    if (sf::once_per_device(attr_done)) {
        // Three prep CTAs share an SM only with the whole unified L1 / shared array as shared memory.
        cudaFuncSetAttribute(kda_prep_kernel<__half, TASK>, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM);
        cudaFuncSetAttribute(kda_prep_kernel<__nv_bfloat16, TASK>, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM);
        cudaFuncSetAttribute(kda_prep_kernel<__half, TASK>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
        cudaFuncSetAttribute(kda_prep_kernel<__nv_bfloat16, TASK>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
        cudaFuncSetAttribute(kda_chain_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, CHAIN_SMEM);
        cudaFuncSetAttribute(kda_chain_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, CHAIN_SMEM);
    }
    int32_t* base = static_cast<int32_t*>(workspace);
    uint8_t* slots = static_cast<uint8_t*>(workspace) + header_bytes(N);
    const int32_t* cu = static_cast<const int32_t*>(cu_seqlens);
    kda_slots_kernel<<<1, 1024, 0, st>>>(cu, (int)N, total_tokens, base, status);
    if (nslots > 0) {
        // [T, H, D] views of q, k (boxes of 64 channels) and g (64 channels of 16-bit gates for the
        // task op, else 32 channels of fp32 log-decay) x one head x 32 tokens.
        const bool bf16 = dtype == SF_DTYPE_BF16;
        CUtensorMap tq, tk, tg;
        int rc = sf::tmap_3d(&tq, q, D, H, total_tokens, D * 2, H * D * 2, 64, 1, C, bf16, err, cap);
        if (rc == SF_OK) rc = sf::tmap_3d(&tk, k, D, H, total_tokens, D * 2, H * D * 2, 64, 1, C, bf16, err, cap);
        if (rc == SF_OK)
            rc = TASK ? sf::tmap_3d(&tg, g, D, H, total_tokens, D * 2, H * D * 2, 64, 1, C, bf16, err, cap)
                      : sf::tmap_3d_f32(&tg, g, D, H, total_tokens, D * 4, H * D * 4, 32, 1, C, err, cap);
        if (rc != SF_OK) return rc;
        if (dtype == SF_DTYPE_F16)
            kda_prep_kernel<__half, TASK><<<(unsigned)nslots, P_NT, PREP_SMEM, st>>>(
                tq, tk, tg, (const __half*)q, (const __half*)k, beta, cu, base, (int)N, nslots, scale, task, (int)H, slots, status);
        else
            kda_prep_kernel<__nv_bfloat16, TASK><<<(unsigned)nslots, P_NT, PREP_SMEM, st>>>(
                tq, tk, tg, (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, beta, cu, base, (int)N, nslots, scale, task, (int)H,
                slots, status);
    }
    if (dtype == SF_DTYPE_F16)
        kda_chain_kernel<__half><<<(unsigned)(N * H), K_NT, CHAIN_SMEM, st>>>((const __half*)v, cu, base, (int)N, nslots,
                                                                              (const float*)initial_state, (int)H, slots, (__half*)out,
                                                                              (float*)final_state, status);
    else
        kda_chain_kernel<__nv_bfloat16><<<(unsigned)(N * H), K_NT, CHAIN_SMEM, st>>>(
            (const __nv_bfloat16*)v, cu, base, (int)N, nslots, (const float*)initial_state, (int)H, slots, (__nv_bfloat16*)out,
            (float*)final_state, status);
    return sf::check_launch(TASK ? "kda two-pass launch" : "kda_gated two-pass launch", err, cap);
}

}  // namespace

// The two-pass kernels; SF_EINVAL (without launching) when the shape, alignment or workspace does
// not qualify.
int sf_kda_gated_split_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                              const void* initial_state, void* out, void* final_state, int64_t N, int64_t total_tokens, int64_t H,
                              int64_t Dd, float scale, int32_t dtype, void* workspace, uint64_t workspace_bytes, cudaStream_t st,
                              char* err, uint64_t cap) {
    return split_launch<false>(q, k, v, g, beta, cu_seqlens, initial_state, out, final_state, N, total_tokens, H, Dd, scale,
                               TaskGate{nullptr, nullptr, nullptr, 0.f}, dtype, workspace, workspace_bytes, st, err, cap);
}

// The task op (in-op q/k norms, gates from A_log / dt_bias, sigmoid beta, an initial state) on the
// two-pass kernels; same qualification rules and workspace.
int sf_kda_task_split_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
                             const void* dt_bias, const void* initial_state, const void* cu_seqlens, const void* scale, void* out,
                             void* final_state, int64_t N, int64_t total_tokens, int64_t H, int64_t Dd, float lower_bound,
                             int32_t dtype, void* workspace, uint64_t workspace_bytes, cudaStream_t st, char* err, uint64_t cap) {
    if (!a_log || !dt_bias || !scale || !initial_state) return sf::fail(SF_EINVAL, err, cap, "kda: null gate / scale / state pointer");
    return split_launch<true>(q, k, v, g, beta, cu_seqlens, initial_state, out, final_state, N, total_tokens, H, Dd, 0.f,
                              TaskGate{(const float*)a_log, (const float*)dt_bias, (const float*)scale, lower_bound}, dtype, workspace,
                              workspace_bytes, st, err, cap);
}

int sf_kda_split_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream) {
    sm100::KernelStatus hs{0, 0};
    if (cudaMemcpyFromSymbolAsync(&hs, g_kda_split_status, sizeof(hs), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess) return SF_EDEVICE;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return SF_EDEVICE;
    if (hs.code) {
        const sm100::KernelStatus zero{0, 0};
        cudaMemcpyToSymbolAsync(g_kda_split_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream);
        cudaStreamSynchronize(stream);
    }
    *code = hs.code;
    *where = hs.where;
    return SF_OK;
}
