// Packed-varlen Kimi Delta Attention (gated delta rule) forward for sm_100a.
//
// Per sequence s (tokens [cu[s], cu[s+1])) and head h, with an fp32 state S [Dv, Dk] (V-first):
//   S <- S * diag(exp(ld_t))                      (decay along the key axis)
//   r  = (v_t - S k_t) * b_t                      (delta residual)
//   S <- S + r k_t^T
//   o_t = S q_t
// Task contract (tasks/varlen_kda/reference.py:323-374): q, k are L2-normalised in-op
// (rsqrt(sum x^2 + 1e-6)), q times `scale`; ld = LOWER_BOUND * sigmoid(exp(A_log[h]) * (g + dt_bias));
// b = sigmoid(beta); S starts from initial_state[s]; final_state[s] = S at the segment end.
// Gated workload: q, k arrive normalised, g is the fp32 log-decay used directly, beta is already
// a gate in (0,1), q times `scale`, S starts at zero (or a given initial state).
//
// Parallel structure: the recurrence never mixes state rows (each row v evolves from k, q, ld, b
// and v_t[v] alone), so a (sequence, head) chain is split over CTAs of 16 state rows each.  A
// CTA has 128 threads: 8 per row, each holding D/8 key columns of the row in registers (thread
// part p owns columns p, p+8, ..., so staged rows are read without bank conflicts).  Per token
// both row dot products of the decayed state S' (S'.k and S'.q) come from one pass and share
// their 3-shuffle reductions over those 8 threads; the output is S_new.q = S'.q + r (k.q), so the
// token-to-token chain carries one reduction.  Tokens are staged 16 at a time in shared memory
// (normalised q/k, their dot product k.q, exp(ld), b, this CTA's v slice) by all
// threads, then consumed sequentially; outputs are staged and written 16 tokens at a time.
// Sentinel offsets (cu < 0, the L2 capacity padding) end the sequence list: such sequences and
// their final_state rows are left untouched.
#include "sf_common.cuh"

#include <type_traits>

namespace {

constexpr int VR = 16;       // state rows per CTA
constexpr int TPR = 8;       // threads per row
constexpr int TS = 16;       // tokens staged per group
constexpr int NT = VR * TPR; // 128 threads

template <typename T, int D, bool TASK>
__global__ void __launch_bounds__(NT) kda_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                                                     const void* __restrict__ g_, const void* __restrict__ beta_,
                                                     const float* __restrict__ a_log, const float* __restrict__ dt_bias,
                                                     const float* __restrict__ state0, const int32_t* __restrict__ cu,
                                                     const float* __restrict__ scale_ptr, float scale_val, float lower_bound, int H,
                                                     T* __restrict__ out, float* __restrict__ final_state) {
    constexpr int CPT = D / TPR;  // key columns per thread
    __shared__ float ks[TS][D];
    __shared__ float qs[TS][D];
    __shared__ float es[TS][D];
    __shared__ float bs[TS];
    __shared__ float kqs[TS];  // k.q of each staged token (normalised and scaled as staged)
    __shared__ float vs[TS][VR];
    __shared__ float os[TS][VR];

    const int chain = blockIdx.x;  // s * H + h
    const int s = chain / H, h = chain % H;
    const int v0 = blockIdx.y * VR;
    const int tid = threadIdx.x;
    const int row = tid / TPR;  // local state row
    const int part = tid % TPR;  // owns key columns part, part + 8, part + 16, ...
    const int vrow = v0 + row;
    const bool row_live = vrow < D;

    const int begin = cu[s];
    const int end = cu[s + 1];
    if (begin < 0 || end < 0 || end < begin) return;  // sentinel: not part of this batch

    const float scale = scale_ptr ? scale_ptr[0] : scale_val;
    float st[CPT];
    const size_t sbase = (((size_t)s * H + h) * D + (row_live ? vrow : 0)) * D + part;
#pragma unroll
    for (int c = 0; c < CPT; ++c) st[c] = (state0 && row_live) ? state0[sbase + (size_t)c * TPR] : 0.f;

    // Staging layout: thread = (token tt = tid / 8, lane-part p = tid % 8) covering D/8 columns.
    // The raw inputs of the next 16-token group are loaded into registers in their storage
    // types before the current group is consumed, so their global-memory latency overlaps the
    // sequential per-token work; they are converted and transformed into shared memory only
    // after that group's tokens are done.
    using GT = typename std::conditional<TASK, T, float>::type;  // storage type of g and beta
    const int stt = tid / TPR;
    const int sp = tid % TPR;
    float decay_scale = 0.f;
    if (TASK) decay_scale = __expf(a_log[h]);
    float dtb[CPT];
#pragma unroll
    for (int c = 0; c < CPT; ++c) dtb[c] = TASK ? dt_bias[h * D + sp + c * TPR] : 0.f;

    const T zt = sf::Dt<T>::from_f(0.f);
    GT zg;
    if constexpr (TASK) zg = zt;
    else zg = 0.f;
    T rq[CPT], rk[CPT], rv[VR / TPR];
    GT rg[CPT], rb = zg;
    auto load_group = [&](int t0) {
        const int t = t0 + stt;
        const bool live = t < end;
        const size_t base = ((size_t)(live ? t : begin) * H + h) * D + sp;
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
            rq[c] = live ? q[base + (size_t)c * TPR] : zt;
            rk[c] = live ? k[base + (size_t)c * TPR] : zt;
            rg[c] = live ? reinterpret_cast<const GT*>(g_)[base + (size_t)c * TPR] : zg;
        }
        if (sp == 0) rb = live ? reinterpret_cast<const GT*>(beta_)[(size_t)t * H + h] : zg;
#pragma unroll
        for (int i = 0; i < VR / TPR; ++i) {
            const int r = sp * (VR / TPR) + i;
            rv[i] = (live && v0 + r < D) ? v[((size_t)t * H + h) * D + v0 + r] : zt;
        }
    };
    auto to_f = [](auto x) -> float {
        if constexpr (std::is_same<decltype(x), float>::value) return x;
        else return sf::Dt<T>::to_f(x);
    };
    if (begin < end) load_group(begin);

    for (int t0 = begin; t0 < end; t0 += TS) {
        const int nt = min(TS, end - t0);
        __syncthreads();  // previous group fully consumed
        {
            const bool live = stt < nt;
            float qv[CPT], kv[CPT];
            float qq = 0.f, kk = 0.f, kq = 0.f;
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                qv[c] = live ? sf::Dt<T>::to_f(rq[c]) : 0.f;
                kv[c] = live ? sf::Dt<T>::to_f(rk[c]) : 0.f;
                qq = fmaf(qv[c], qv[c], qq);
                kk = fmaf(kv[c], kv[c], kk);
                kq = fmaf(kv[c], qv[c], kq);
            }
#pragma unroll
            for (int o = 1; o < TPR; o <<= 1) kq += __shfl_xor_sync(0xffffffffu, kq, o);
            float qn = scale, kn = 1.f;
            if (TASK) {
#pragma unroll
                for (int o = 1; o < TPR; o <<= 1) {
                    qq += __shfl_xor_sync(0xffffffffu, qq, o);
                    kk += __shfl_xor_sync(0xffffffffu, kk, o);
                }
                qn = rsqrtf(qq + 1e-6f) * scale;
                kn = rsqrtf(kk + 1e-6f);
            }
#pragma unroll
            for (int c = 0; c < CPT; ++c) {
                const int col = sp + c * TPR;
                qs[stt][col] = qv[c] * qn;
                ks[stt][col] = kv[c] * kn;
                float e = 1.f;
                if (live) {
                    if (TASK) {
                        const float z = decay_scale * (to_f(rg[c]) + dtb[c]);
                        const float ld = lower_bound / (1.f + __expf(-z));
                        e = __expf(ld);
                    } else {
                        e = __expf(to_f(rg[c]));
                    }
                }
                es[stt][col] = e;
            }
            if (sp == 0) {
                float b = 0.f;
                if (live) b = TASK ? 1.f / (1.f + __expf(-to_f(rb))) : to_f(rb);
                bs[stt] = b;
                kqs[stt] = kq * kn * qn;
            }
            // v slice: VR rows of token stt, threads sp 0..7 cover VR columns (2 each).
#pragma unroll
            for (int i = 0; i < VR / TPR; ++i) {
                const int r = sp * (VR / TPR) + i;
                vs[stt][r] = (live && v0 + r < D) ? sf::Dt<T>::to_f(rv[i]) : 0.f;
            }
        }
        __syncthreads();
        if (t0 + TS < end) load_group(t0 + TS);
#pragma unroll 4
        for (int tt = 0; tt < nt; ++tt) {
            // One pass over the decayed state S' gives both S'.k and S'.q; the output is then
            // S_new.q = S'.q + r (k.q) with k.q staged per token, so the only dependent reduction
            // on the token-to-token chain is S'.k (the two reductions share their shuffle levels).
            float acc0 = 0.f, acc1 = 0.f, oq0 = 0.f, oq1 = 0.f;
#pragma unroll
            for (int c = 0; c < CPT; c += 2) {
                st[c] *= es[tt][part + c * TPR];
                acc0 = fmaf(st[c], ks[tt][part + c * TPR], acc0);
                oq0 = fmaf(st[c], qs[tt][part + c * TPR], oq0);
                if (c + 1 < CPT) {
                    st[c + 1] *= es[tt][part + (c + 1) * TPR];
                    acc1 = fmaf(st[c + 1], ks[tt][part + (c + 1) * TPR], acc1);
                    oq1 = fmaf(st[c + 1], qs[tt][part + (c + 1) * TPR], oq1);
                }
            }
            float acc = acc0 + acc1, oq = oq0 + oq1;
#pragma unroll
            for (int o = 1; o < TPR; o <<= 1) {
                acc += __shfl_xor_sync(0xffffffffu, acc, o);
                oq += __shfl_xor_sync(0xffffffffu, oq, o);
            }
            const float r = (vs[tt][row] - acc) * bs[tt];
#pragma unroll
            for (int c = 0; c < CPT; ++c) st[c] = fmaf(r, ks[tt][part + c * TPR], st[c]);
            if (part == 0) os[tt][row] = fmaf(r, kqs[tt], oq);
        }
        __syncthreads();
        // Write the group's outputs: token-major, VR contiguous values per token.
        for (int i = tid; i < nt * VR; i += NT) {
            const int tt = i / VR, r = i % VR;
            if (v0 + r < D) out[((size_t)(t0 + tt) * H + h) * D + v0 + r] = sf::Dt<T>::from_f(os[tt][r]);
        }
    }
    if (row_live) {
#pragma unroll
        for (int c = 0; c < CPT; ++c) final_state[sbase + (size_t)c * TPR] = st[c];
    }
}

template <typename T, bool TASK>
int launch_t(const void* q, const void* k, const void* v, const void* g, const void* beta, const float* a_log, const float* dt_bias,
             const float* state0, const int32_t* cu, const float* scale_ptr, float scale_val, float lower_bound, int64_t N, int64_t H,
             int64_t D, void* out, float* final_state, cudaStream_t st, char* err, uint64_t cap) {
    const dim3 grid((unsigned)(N * H), (unsigned)((D + VR - 1) / VR));
#define SF_KDA_CASE(DD)                                                                                                        \
    case DD:                                                                                                                   \
        kda_fwd_kernel<T, DD, TASK><<<grid, NT, 0, st>>>((const T*)q, (const T*)k, (const T*)v, g, beta, a_log, dt_bias, state0, \
                                                        cu, scale_ptr, scale_val, lower_bound, (int)H, (T*)out, final_state); \
        break;
    switch (D) {
        SF_KDA_CASE(8)
        SF_KDA_CASE(16)
        SF_KDA_CASE(32)
        SF_KDA_CASE(64)
        SF_KDA_CASE(128)
        default:
            return sf::fail(SF_EINVAL, err, cap, "kda: head dim %lld is not one of 8/16/32/64/128", (long long)D);
    }
#undef SF_KDA_CASE
    return sf::check_launch("kda launch", err, cap);
}

int check(int64_t N, int64_t H, int64_t D, int32_t dtype, char* err, uint64_t cap) {
    if (N < 0 || H < 1 || D < 1) return sf::fail(SF_EINVAL, err, cap, "kda: need num_seqs >= 0, H >= 1, D >= 1");
    if (dtype != SF_DTYPE_F16 && dtype != SF_DTYPE_BF16) return sf::fail(SF_EINVAL, err, cap, "kda: dtype %d is not fp16/bf16", dtype);
    if (N * H > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "kda: too many chains");
    return SF_OK;
}

}  // namespace

int sf_kda_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log, const void* dt_bias,
                  const void* initial_state, const void* cu_seqlens, const void* scale, void* out, void* final_state, int64_t N,
                  int64_t H, int64_t D, float lower_bound, int32_t dtype, int32_t variant, int64_t total_tokens, void* workspace,
                  uint64_t workspace_bytes, cudaStream_t st, char* err, uint64_t cap) {
    int rc = check(N, H, D, dtype, err, cap);
    if (rc) return rc;
    if (N == 0) return SF_OK;
    if (!q || !k || !v || !g || !beta || !a_log || !dt_bias || !initial_state || !cu_seqlens || !scale || !out || !final_state)
        return sf::fail(SF_EINVAL, err, cap, "kda: null tensor pointer");
    // Variant 0: the two-pass kernels (all 32-token chunks prepared in parallel, then the chains)
    // when they apply (D = 128, aligned rows, a workspace of sf_varlen_kda_workspace_bytes), else
    // the 16-token chunked kernel (D = 128, aligned rows), else the recurrent one.  4 forces the
    // two-pass kernels, 1 the 16-token chunked kernel, 2 the recurrent one.
    if (variant == 4 || (variant == 0 && workspace)) {
        rc = sf_kda_task_split_launch(q, k, v, g, beta, a_log, dt_bias, initial_state, cu_seqlens, scale, out, final_state, N,
                                      total_tokens, H, D, lower_bound, dtype, workspace, workspace_bytes, st,
                                      variant == 4 ? err : nullptr, variant == 4 ? cap : 0);
        if (rc == SF_OK || variant == 4 || rc != SF_EINVAL) return rc;
    }
    if (variant != 2) {
        rc = sf_kda_task_chunk_launch(q, k, v, g, beta, a_log, dt_bias, initial_state, cu_seqlens, scale, out, final_state, N, H, D,
                                      lower_bound, dtype, st, variant == 1 ? err : nullptr, variant == 1 ? cap : 0);
        if (rc == SF_OK || variant == 1 || rc != SF_EINVAL) return rc;
    }
    if (dtype == SF_DTYPE_F16)
        return launch_t<__half, true>(q, k, v, g, beta, (const float*)a_log, (const float*)dt_bias, (const float*)initial_state,
                                      (const int32_t*)cu_seqlens, (const float*)scale, 0.f, lower_bound, N, H, D, out,
                                      (float*)final_state, st, err, cap);
    return launch_t<__nv_bfloat16, true>(q, k, v, g, beta, (const float*)a_log, (const float*)dt_bias, (const float*)initial_state,
                                         (const int32_t*)cu_seqlens, (const float*)scale, 0.f, lower_bound, N, H, D, out,
                                         (float*)final_state, st, err, cap);
}

int sf_kda_gated_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                        const void* initial_state, void* out, void* final_state, int64_t N, int64_t H, int64_t D, float scale,
                        int32_t dtype, int32_t variant, int64_t total_tokens, void* workspace, uint64_t workspace_bytes,
                        cudaStream_t st, char* err, uint64_t cap) {
    int rc = check(N, H, D, dtype, err, cap);
    if (rc) return rc;
    if (N == 0) return SF_OK;
    if (!q || !k || !v || !g || !beta || !cu_seqlens || !out || !final_state)
        return sf::fail(SF_EINVAL, err, cap, "kda_gated: null tensor pointer");
    // Variant 0: the two-pass kernels (all chunks prepared in parallel, then the chains) when
    // they apply (D = 128, aligned rows, a workspace of sf_varlen_kda_gated_workspace_bytes),
    // else the single-pass 32-token kernel, else the recurrent one.  4 forces the two-pass
    // kernels, 1 the single-pass 32-token kernel, 3 the 16-token kernel, 2 the recurrent kernel.
    if (variant == 4 || (variant == 0 && workspace)) {
        rc = sf_kda_gated_split_launch(q, k, v, g, beta, cu_seqlens, initial_state, out, final_state, N, total_tokens, H, D, scale, dtype,
                                       workspace, workspace_bytes, st, variant == 4 ? err : nullptr, variant == 4 ? cap : 0);
        if (rc == SF_OK || variant == 4 || rc != SF_EINVAL) return rc;
    }
    if (variant == 3)
        return sf_kda_gated_chunk_launch(q, k, v, g, beta, cu_seqlens, initial_state, out, final_state, N, H, D, scale, dtype, st, err,
                                         cap);
    if (variant != 2) {
        rc = sf_kda_gated_c32_launch(q, k, v, g, beta, cu_seqlens, initial_state, out, final_state, N, H, D, scale, dtype, st,
                                     variant == 1 ? err : nullptr, variant == 1 ? cap : 0);
        if (rc == SF_OK || variant == 1 || rc != SF_EINVAL) return rc;
    }
    if (dtype == SF_DTYPE_F16)
        return launch_t<__half, false>(q, k, v, g, beta, nullptr, nullptr, (const float*)initial_state, (const int32_t*)cu_seqlens,
                                       nullptr, scale, 0.f, N, H, D, out, (float*)final_state, st, err, cap);
    return launch_t<__nv_bfloat16, false>(q, k, v, g, beta, nullptr, nullptr, (const float*)initial_state, (const int32_t*)cu_seqlens,
                                          nullptr, scale, 0.f, N, H, D, out, (float*)final_state, st, err, cap);
}

namespace {

// Host program of the fixed-length task: the single sequence is one work item [0, N) (the
// reference's work list holds at most three [token_begin, token_count] pieces; one piece covers
// any N here because the recurrence runs inside one launch).  Rows 1 and 2 are empty [N, 0) items.
__global__ void kda_fixed_items_kernel(uint32_t* __restrict__ work_items, int32_t* __restrict__ item_counts, uint32_t n) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        work_items[0] = 0u;
        work_items[1] = n;
        work_items[2] = n;
        work_items[3] = 0u;
        work_items[4] = n;
        work_items[5] = 0u;
        item_counts[0] = 1;
    }
}

}  // namespace

// Fixed-length KDA (tasks/kda/reference.py reference()): the varlen recurrence over one sequence of
// N tokens.  work_items row 0 = (0, N) read as int32 is exactly the cu_seqlens [0, N] of that one
// sequence, so the kernel takes it directly and nothing is allocated.  handoff_states (the state
// at piece boundaries when the work is cut into several pieces) is not written: one piece has no
// boundary.
int sf_kda_fixed_launch(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
                        const void* dt_bias, const void* initial_state, const void* scale, void* out, void* final_state,
                        void* work_items, void* item_counts, int64_t N, int64_t H, int64_t D, float lower_bound, int32_t dtype,
                        int32_t variant, cudaStream_t st, char* err, uint64_t cap) {
    int rc = check(1, H, D, dtype, err, cap);
    if (rc) return rc;
    if (N < 0 || N > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "kda: N=%lld out of range", (long long)N);
    if (!work_items || !item_counts) return sf::fail(SF_EINVAL, err, cap, "kda: null work_items / item_counts");
    if (reinterpret_cast<uintptr_t>(work_items) & 3u) return sf::fail(SF_EINVAL, err, cap, "kda: work_items is not 4-byte aligned");
    kda_fixed_items_kernel<<<1, 32, 0, st>>>((uint32_t*)work_items, (int32_t*)item_counts, (uint32_t)N);
    rc = sf::check_launch("kda work-list launch", err, cap);
    if (rc) return rc;
    // Default: the recurrent fp32 kernel at every D.  The chunked kernel's TF32 products meet
    // varlen_kda's tolerance but not always this task's tighter one (fp16 rtol 2e-3 / atol_rel
    // 1e-3): at D = 128 one output in 76,800 of the wide_range case landed at 1.15x the bound.
    // variant 1 still forces the chunked kernel.
    return sf_kda_launch(q, k, v, g, beta, a_log, dt_bias, initial_state, work_items, scale, out, final_state, 1, H, D, lower_bound,
                         dtype, variant == 1 ? 1 : 2, 0, nullptr, 0, st, err, cap);
}

extern "C" int sf_kda(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
                      const void* dt_bias, const void* initial_state, const void* scale, void* output, void* final_state,
                      void* work_items, void* item_counts, void* handoff_states, int64_t N, int64_t H, int64_t D, float lower_bound,
                      int32_t dtype, void* stream, char* err, uint64_t cap) {
    (void)handoff_states;
    return sf_kda_fixed_launch(q, k, v, g, beta, a_log, dt_bias, initial_state, scale, output, final_state, work_items, item_counts,
                               N, H, D, lower_bound, dtype, 0, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_varlen_kda(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
                             const void* dt_bias, const void* initial_state, const void* cu_seqlens, const void* scale, void* output,
                             void* final_state, int64_t num_seqs, int64_t H, int64_t D, float lower_bound, int32_t dtype, void* stream,
                             char* err, uint64_t cap) {
    return sf_kda_launch(q, k, v, g, beta, a_log, dt_bias, initial_state, cu_seqlens, scale, output, final_state, num_seqs, H, D,
                         lower_bound, dtype, 0, 0, nullptr, 0, (cudaStream_t)stream, err, cap);
}

extern "C" uint64_t sf_varlen_kda_workspace_bytes(int64_t total_tokens, int64_t num_seqs, int64_t H, int64_t D) {
    return sf_kda_gated_split_workspace(total_tokens, num_seqs, H, D);
}

extern "C" int sf_varlen_kda_ws(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
                                const void* dt_bias, const void* initial_state, const void* cu_seqlens, const void* scale, void* output,
                                void* final_state, int64_t num_seqs, int64_t total_tokens, int64_t H, int64_t D, float lower_bound,
                                int32_t dtype, void* workspace, uint64_t workspace_bytes, void* stream, char* err, uint64_t cap) {
    return sf_kda_launch(q, k, v, g, beta, a_log, dt_bias, initial_state, cu_seqlens, scale, output, final_state, num_seqs, H, D,
                         lower_bound, dtype, 0, total_tokens, workspace, workspace_bytes, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_varlen_kda_gated(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* cu_seqlens,
                                   const void* initial_state, void* output, void* final_state, int64_t num_seqs, int64_t H, int64_t D,
                                   float scale, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_kda_gated_launch(q, k, v, g, beta, cu_seqlens, initial_state, output, final_state, num_seqs, H, D, scale, dtype, 0, 0,
                               nullptr, 0, (cudaStream_t)stream, err, cap);
}

extern "C" uint64_t sf_varlen_kda_gated_workspace_bytes(int64_t total_tokens, int64_t num_seqs, int64_t H, int64_t D) {
    return sf_kda_gated_split_workspace(total_tokens, num_seqs, H, D);
}

extern "C" int sf_varlen_kda_gated_ws(const void* q, const void* k, const void* v, const void* g, const void* beta,
                                      const void* cu_seqlens, const void* initial_state, void* output, void* final_state,
                                      int64_t num_seqs, int64_t total_tokens, int64_t H, int64_t D, float scale, int32_t dtype,
                                      void* workspace, uint64_t workspace_bytes, void* stream, char* err, uint64_t cap) {
    return sf_kda_gated_launch(q, k, v, g, beta, cu_seqlens, initial_state, output, final_state, num_seqs, H, D, scale, dtype, 0,
                               total_tokens, workspace, workspace_bytes, (cudaStream_t)stream, err, cap);
}
