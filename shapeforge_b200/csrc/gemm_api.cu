// GEMM entry points of the C ABI and their general-shape fallback.
//
//   sf_gemm_nt  C = A . B^T, B stored [N, K]  (the dense-gemm workload's layout)
//   sf_gemm_nn  C = A . B,   B stored [K, N]  (tasks/gemm/reference.py:110-114)
//   sf_gemm_silu C = silu(A . B), B stored [K, N] (tasks/gemm_silu/reference.py), same dispatch
//
// Dispatch mirrors the reference portfolio's exact one-of-N + fallback rule
// (tcenv/portfolio/dispatch.py:595-700): the tcgen05 kernel (gemm_tc.cu) serves every shape it
// supports (16-byte aligned bases, K % 8 == 0); everything else runs the general fallback below,
// a tiled fp32-accumulate SIMT kernel valid for any M, N, K >= 0 and any alignment.  The NN
// layout is read by the tensor-core kernel directly (B as an MN-major operand) when N % 8 == 0;
// otherwise it goes through a transpose of B into a caller-provided workspace of K*N elements
// (sf_gemm_nn_workspace_bytes, 0 when no workspace is needed), and without one takes the fallback.
#include "sf_common.cuh"

#include <algorithm>

bool sf_gemm_nt_tc_supported(const void* A, const void* B, const void* C, int64_t M, int64_t N, int64_t K);
int sf_gemm_nt_tc_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, bool silu,
                         cudaStream_t stream, char* err, uint64_t cap);
int sf_gemm_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream);
bool sf_gemm_nn_tc_supported(const void* A, const void* B, const void* C, int64_t M, int64_t N, int64_t K);
int sf_gemm_nn_tc_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, bool silu,
                         cudaStream_t stream, char* err, uint64_t cap);

namespace {

constexpr int FB_BM = 64, FB_BN = 64, FB_BK = 16;

// B_KN = true: B is [K, N] (NN); false: B is [N, K] (NT).  SILU = true stores acc * sigmoid(acc).
template <typename T, bool B_KN, bool SILU>
__global__ void __launch_bounds__(256) gemm_fallback_kernel(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C,
                                                            int64_t M, int64_t N, int64_t K) {
    __shared__ float As[FB_BK][FB_BM + 1];
    __shared__ float Bs[FB_BK][FB_BN + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * FB_BM, n0 = (int64_t)blockIdx.x * FB_BN;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < K; k0 += FB_BK) {
        for (int i = threadIdx.x; i < FB_BM * FB_BK; i += 256) {
            const int r = i / FB_BK, c = i % FB_BK;
            const int64_t gm = m0 + r, gk = k0 + c;
            As[c][r] = (gm < M && gk < K) ? sf::Dt<T>::to_f(A[gm * K + gk]) : 0.f;
        }
        for (int i = threadIdx.x; i < FB_BN * FB_BK; i += 256) {
            int r, c;
            if (B_KN) {
                c = i / FB_BN;
                r = i % FB_BN;  // consecutive threads read consecutive n
            } else {
                r = i / FB_BK;
                c = i % FB_BK;
            }
            const int64_t gn = n0 + r, gk = k0 + c;
            float v = 0.f;
            if (gn < N && gk < K) v = sf::Dt<T>::to_f(B_KN ? B[gk * N + gn] : B[gn * K + gk]);
            Bs[c][r] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < FB_BK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t gm = m0 + ty + 16 * i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t gn = n0 + tx + 16 * j;
            float v = acc[i][j];
            if (SILU) v = v * sf::sigmoid_nr(v);
            if (gn < N) C[gm * N + gn] = sf::Dt<T>::from_f(v);
        }
    }
}

template <typename T, bool B_KN, bool SILU>
int launch_fallback_t(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, cudaStream_t s, char* err,
                      uint64_t cap) {
    const int64_t gx = (N + FB_BN - 1) / FB_BN, gy = (M + FB_BM - 1) / FB_BM;
    if (gy > 65535) return sf::fail(SF_EINVAL, err, cap, "gemm fallback: M=%lld too large", (long long)M);
    gemm_fallback_kernel<T, B_KN, SILU><<<dim3((unsigned)gx, (unsigned)gy), 256, 0, s>>>((const T*)A, (const T*)B, (T*)C, M, N, K);
    return sf::check_launch("gemm fallback launch", err, cap);
}

template <bool B_KN>
int launch_fallback(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, bool silu,
                    cudaStream_t s, char* err, uint64_t cap) {
    if (dtype == SF_DTYPE_F16)
        return silu ? launch_fallback_t<__half, B_KN, true>(A, B, C, M, N, K, s, err, cap)
                    : launch_fallback_t<__half, B_KN, false>(A, B, C, M, N, K, s, err, cap);
    if (dtype == SF_DTYPE_BF16)
        return silu ? launch_fallback_t<__nv_bfloat16, B_KN, true>(A, B, C, M, N, K, s, err, cap)
                    : launch_fallback_t<__nv_bfloat16, B_KN, false>(A, B, C, M, N, K, s, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "gemm: dtype %d is not fp16/bf16", dtype);
}

// [K, N] -> [N, K] transpose of 16-bit elements through a 64x64 shared tile (coalesced both ways).
__global__ void __launch_bounds__(256) transpose16_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst,
                                                          int64_t rows, int64_t cols) {
    __shared__ uint16_t tile[64][65];
    const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
    const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4
    for (int i = ty; i < 64; i += 4) {
        const int64_t r = r0 + i, c = c0 + tx;
        if (r < rows && c < cols) tile[i][tx] = src[r * cols + c];
    }
    __syncthreads();
    for (int i = ty; i < 64; i += 4) {
        const int64_t c = c0 + i, r = r0 + tx;  // dst[c, r]
        if (c < cols && r < rows) dst[c * rows + r] = tile[tx][i];
    }
}

int check_common(const void* A, const void* B, const void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, char* err,
                 uint64_t cap) {
    if (M < 0 || N < 0 || K < 0) return sf::fail(SF_EINVAL, err, cap, "gemm: negative size");
    if (dtype != SF_DTYPE_F16 && dtype != SF_DTYPE_BF16) return sf::fail(SF_EINVAL, err, cap, "gemm: dtype %d is not fp16/bf16", dtype);
    if (M > 0 && N > 0) {
        if (!C) return sf::fail(SF_EINVAL, err, cap, "gemm: null output pointer");
        if (K > 0 && (!A || !B)) return sf::fail(SF_EINVAL, err, cap, "gemm: null input pointer");
    }
    return SF_OK;
}

__global__ void zero16_kernel(uint16_t* __restrict__ p, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = 0;
}

// K == 0: C is the empty sum, i.e. +0.
int zero_output(void* C, int64_t M, int64_t N, cudaStream_t s, char* err, uint64_t cap) {
    const int64_t n = M * N;
    if (n == 0) return SF_OK;
    zero16_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, s>>>((uint16_t*)C, n);
    return sf::check_launch("gemm zero launch", err, cap);
}

}  // namespace

// variant: 0 = dispatch (tcgen05 when supported, else fallback), 1 = force tcgen05 (error if
// unsupported), 2 = force the general fallback.
int sf_gemm_nt_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, int32_t variant,
                      cudaStream_t s, char* err, uint64_t cap) {
    int rc = check_common(A, B, C, M, N, K, dtype, err, cap);
    if (rc) return rc;
    if (M == 0 || N == 0) return SF_OK;
    if (K == 0) return zero_output(C, M, N, s, err, cap);
    const bool tc = sf_gemm_nt_tc_supported(A, B, C, M, N, K);
    if (variant == 1 && !tc) return sf::fail(SF_EINVAL, err, cap, "gemm_nt: the tcgen05 variant needs 16-byte aligned bases and K %% 8 == 0");
    if (tc && variant != 2) return sf_gemm_nt_tc_launch(A, B, C, M, N, K, dtype, false, s, err, cap);
    return launch_fallback<false>(A, B, C, M, N, K, dtype, false, s, err, cap);
}

namespace {

// C = A . B (silu = false) or C = silu(A . B) (silu = true) with B stored [K, N].
int nn_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, int32_t variant, bool silu,
              void* workspace, uint64_t workspace_bytes, cudaStream_t s, char* err, uint64_t cap) {
    const char* name = silu ? "gemm_silu" : "gemm_nn";
    int rc = check_common(A, B, C, M, N, K, dtype, err, cap);
    if (rc) return rc;
    if (M == 0 || N == 0) return SF_OK;
    // K == 0: the empty sum is +0 and silu(+0) = +0.
    if (K == 0) return zero_output(C, M, N, s, err, cap);
    const bool direct = sf_gemm_nn_tc_supported(A, B, C, M, N, K);
    if (direct && variant != 2) return sf_gemm_nn_tc_launch(A, B, C, M, N, K, dtype, silu, s, err, cap);
    const uint64_t need = (uint64_t)K * (uint64_t)N * 2u;
    const bool ws_ok = workspace && workspace_bytes >= need && sf::aligned16(workspace);
    const bool tc = ws_ok && sf_gemm_nt_tc_supported(A, workspace, C, M, N, K);
    if (variant == 1 && !tc)
        return sf::fail(SF_EINVAL, err, cap,
                        "%s: the tcgen05 variant needs aligned bases with N %% 8 == 0, or a 16-byte aligned workspace of %llu bytes; "
                        "and K %% 8 == 0", name, (unsigned long long)need);
    if (tc && variant != 2) {
        const int64_t gx = (N + 63) / 64, gy = (K + 63) / 64;
        if (gy > 65535) return sf::fail(SF_EINVAL, err, cap, "%s: K=%lld too large for the transpose grid", name, (long long)K);
        transpose16_kernel<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, s>>>((const uint16_t*)B, (uint16_t*)workspace, K, N);
        rc = sf::check_launch("gemm_nn transpose launch", err, cap);
        if (rc) return rc;
        return sf_gemm_nt_tc_launch(A, workspace, C, M, N, K, dtype, silu, s, err, cap);
    }
    return launch_fallback<true>(A, B, C, M, N, K, dtype, silu, s, err, cap);
}

}  // namespace

int sf_gemm_nn_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, int32_t variant,
                      void* workspace, uint64_t workspace_bytes, cudaStream_t s, char* err, uint64_t cap) {
    return nn_launch(A, B, C, M, N, K, dtype, variant, false, workspace, workspace_bytes, s, err, cap);
}

// gemm_silu (tasks/gemm_silu/reference.py): the gemm_nn dispatch with the SiLU epilogue fused
// into whichever kernel runs (tcgen05 direct, tcgen05 after the workspace transpose, or fallback).
int sf_gemm_silu_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, int32_t variant,
                        void* workspace, uint64_t workspace_bytes, cudaStream_t s, char* err, uint64_t cap) {
    return nn_launch(A, B, C, M, N, K, dtype, variant, true, workspace, workspace_bytes, s, err, cap);
}


extern "C" int sf_gemm_nt(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, void* stream,
                          char* err, uint64_t cap) {
    return sf_gemm_nt_launch(A, B, C, M, N, K, dtype, 0, (cudaStream_t)stream, err, cap);
}

extern "C" uint64_t sf_gemm_nn_workspace_bytes(int64_t M, int64_t N, int64_t K, int32_t dtype) {
    (void)M;
    (void)dtype;
    // N % 8 == 0 (with 16-byte aligned tensors) runs without a workspace.
    if (N <= 0 || K <= 0 || N % 8 == 0) return 0;
    return (uint64_t)N * (uint64_t)K * 2u;
}

extern "C" int sf_gemm_nn(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, void* workspace,
                          uint64_t workspace_bytes, void* stream, char* err, uint64_t cap) {
    return sf_gemm_nn_launch(A, B, C, M, N, K, dtype, 0, workspace, workspace_bytes, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_gemm_silu(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, void* workspace,
                            uint64_t workspace_bytes, void* stream, char* err, uint64_t cap) {
    return sf_gemm_silu_launch(A, B, C, M, N, K, dtype, 0, workspace, workspace_bytes, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_kernel_status(uint32_t* code, uint32_t* where, void* stream, char* err, uint64_t cap) {
    if (!code || !where) return sf::fail(SF_EINVAL, err, cap, "sf_kernel_status: null output");
    // Each tensor-core module keeps its own status word; the first failure found is reported
    // (the wait ids are unique across modules) and every word is cleared.
    uint32_t c[7] = {0, 0, 0, 0, 0, 0, 0}, w[7] = {0, 0, 0, 0, 0, 0, 0};
    if (sf_gemm_status_read(&c[0], &w[0], (cudaStream_t)stream) != SF_OK ||
        sf_bitdelta_status_read(&c[1], &w[1], (cudaStream_t)stream) != SF_OK ||
        sf_attention_status_read(&c[2], &w[2], (cudaStream_t)stream) != SF_OK ||
        sf_mamba2_status_read(&c[3], &w[3], (cudaStream_t)stream) != SF_OK ||
        sf_kda_status_read(&c[4], &w[4], (cudaStream_t)stream) != SF_OK ||
        sf_kda32_status_read(&c[5], &w[5], (cudaStream_t)stream) != SF_OK ||
        sf_kda_split_status_read(&c[6], &w[6], (cudaStream_t)stream) != SF_OK)
        return sf::fail(SF_EDEVICE, err, cap, "sf_kernel_status: reading the status word failed");
    *code = 0;
    *where = 0;
    for (int i = 0; i < 7; ++i) {
        if (c[i] && !*code) {
            *code = c[i];
            *where = w[i];
        }
    }
    return SF_OK;
}
