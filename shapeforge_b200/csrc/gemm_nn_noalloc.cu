// sf_gemm_nn_noalloc: C[M,N] = A[M,K] . B[K,N] without any device allocation.
//
// Who needs this.  sf_gemm_nn reads B in place when N % 8 == 0, but for other N it runs the
// tensor-core kernel on a transposed copy of B, and that copy lives in a workspace the caller
// allocates.  Some callers cannot allocate device memory when they need the product:
//   * hosts whose device memory is entirely reserved up front by another allocator (a caching
//     allocator or a memory pool sized to the card) and that give a plug-in no way into it: a
//     raw cudaMalloc there fails or fragments the pool;
//   * certified or real-time hosts that forbid dynamic allocation after start-up.
// For them this entry point keeps the transpose scratch in a fixed, file-scope device array.
// It makes CUDA API calls (device query, symbol lookup, kernel launches), so like every entry
// point of this library it must not be called from a host function or stream callback
// (cudaLaunchHostFunc), where CUDA API calls are not permitted.
//
// Dispatch is sf_gemm_nn's, with the array standing in for the caller workspace:
//   * N % 8 == 0 with 16-byte aligned tensors and K % 8 == 0: the tensor-core kernel reads B in
//     place; the array is not touched and no size limit applies;
//   * otherwise, when the tensor-core kernel can run on a transposed B (K % 8 == 0, aligned A
//     and C): B is transposed into the array first;
//   * otherwise (K % 8 != 0 or misaligned A/C): the general kernel reads B directly, no scratch;
//   * K == 0: C is set to +0.
//
// The price.  The array (SF_GEMM_NN_NOALLOC_MAX_SCRATCH_BYTES = 32 MiB) is reserved on every
// GPU that loads the library, for as long as the process lives.  A problem that needs the
// transpose and whose transposed B (K*N 16-bit elements) does not fit is rejected with
// SF_EINVAL.  All calls on a device share the one array, and it keeps whatever the previous
// call left there; nothing in it needs to start at zero, because every call overwrites the K*N
// elements it reads before reading them.  Calls that overlap on the GPU (on different streams,
// or from several threads without ordering) race on the array and produce wrong results:
// serialise them on one stream.
//
// Set-up.  The first call that needs the array in a CUDA context resolves the array's device
// address with cudaGetSymbolAddress while that context is current, and caches it under the
// context's unique id (cuCtxGetId), so a context created later (after cudaDeviceReset, say)
// resolves its own.  Make that first call before any stream capture begins on the device.  In
// host code the array's name is only a host-side stand-in, never a device address, which is why
// the resolved pointer is what the kernels receive.
#include "sf_common.cuh"

#include <cuda.h>

#include <mutex>

bool sf_gemm_nn_tc_supported(const void* A, const void* B, const void* C, int64_t M, int64_t N, int64_t K);
bool sf_gemm_nt_tc_supported(const void* A, const void* B, const void* C, int64_t M, int64_t N, int64_t K);
int sf_gemm_nt_tc_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, bool silu,
                         cudaStream_t stream, char* err, uint64_t cap);
int sf_gemm_nn_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, int32_t variant,
                      void* workspace, uint64_t workspace_bytes, cudaStream_t s, char* err, uint64_t cap);

// The transpose scratch shared by every call on a device (see above).
static __device__ __align__(256) uint8_t g_gemm_nn_scratch[SF_GEMM_NN_NOALLOC_MAX_SCRATCH_BYTES];

namespace {

constexpr uint64_t kScratchBytes = SF_GEMM_NN_NOALLOC_MAX_SCRATCH_BYTES;
constexpr int kMaxContexts = 64;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

std::mutex g_setup_mu;
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;
unsigned long long g_ctx_ids[kMaxContexts] = {};
void* g_scratch_ptrs[kMaxContexts] = {};
int g_nctx = 0;

// Unique id of the current CUDA context (made current by the runtime if none is yet).
int current_context_id(unsigned long long* id, char* err, uint64_t cap) {
    if (!g_ctx_get_current || !g_ctx_get_id) {
        void* p1 = nullptr;
        void* p2 = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p1, cudaEnableDefault, &q1) != cudaSuccess ||
            q1 != cudaDriverEntryPointSuccess || !p1 ||
            cudaGetDriverEntryPoint("cuCtxGetId", &p2, cudaEnableDefault, &q2) != cudaSuccess ||
            q2 != cudaDriverEntryPointSuccess || !p2)
            return sf::fail(SF_EDEVICE, err, cap, "gemm_nn_noalloc: the driver does not export cuCtxGetCurrent/cuCtxGetId");
        g_ctx_get_current = (CtxGetCurrentFn)p1;
        g_ctx_get_id = (CtxGetIdFn)p2;
    }
    // A context the caller made current (primary or its own) is used as it is.  Only a thread
    // with none gets the current device's primary context, through cudaSetDevice, exactly as the
    // runtime's kernel launches below would bind it.
    CUcontext ctx = nullptr;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) return sf::fail(SF_EDEVICE, err, cap, "gemm_nn_noalloc: cuCtxGetCurrent failed");
    if (!ctx) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaSetDevice(dev);
        if (e != cudaSuccess) return sf::fail(SF_EDEVICE, err, cap, "gemm_nn_noalloc: no CUDA context: %s", cudaGetErrorString(e));
        if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || !ctx)
            return sf::fail(SF_EDEVICE, err, cap, "gemm_nn_noalloc: no current CUDA context");
    }
    if (g_ctx_get_id(ctx, id) != CUDA_SUCCESS) return sf::fail(SF_EDEVICE, err, cap, "gemm_nn_noalloc: cuCtxGetId failed");
    return SF_OK;
}

// Device address of the scratch array in the current context (resolved once per context).
int scratch_for_current_context(void** out, char* err, uint64_t cap) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    unsigned long long id = 0;
    int rc = current_context_id(&id, err, cap);
    if (rc) return rc;
    for (int i = 0; i < g_nctx; ++i) {
        if (g_ctx_ids[i] == id) {
            *out = g_scratch_ptrs[i];
            return SF_OK;
        }
    }
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_gemm_nn_scratch);
    if (e != cudaSuccess || !p)
        return sf::fail(SF_EDEVICE, err, cap, "gemm_nn_noalloc: cudaGetSymbolAddress of the scratch array failed: %s",
                        cudaGetErrorString(e));
    // Contexts past the table's size are resolved on every call (still correct, just slower).
    if (g_nctx < kMaxContexts) {
        g_ctx_ids[g_nctx] = id;
        g_scratch_ptrs[g_nctx] = p;
        ++g_nctx;
    }
    *out = p;
    return SF_OK;
}

// [K, N] -> [N, K] transpose of 16-bit elements through a 64x64 shared tile.
__global__ void __launch_bounds__(256) noalloc_transpose16_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst,
                                                                  int64_t rows, int64_t cols) {
    __shared__ uint16_t tile[64][65];
    const int64_t r0 = (int64_t)blockIdx.y * 64, c0 = (int64_t)blockIdx.x * 64;
    const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;
    for (int i = ty; i < 64; i += 4) {
        const int64_t r = r0 + i, c = c0 + tx;
        if (r < rows && c < cols) tile[i][tx] = src[r * cols + c];
    }
    __syncthreads();
    for (int i = ty; i < 64; i += 4) {
        const int64_t c = c0 + i, r = r0 + tx;
        if (c < cols && r < rows) dst[c * rows + r] = tile[tx][i];
    }
}

}  // namespace

extern "C" int sf_gemm_nn_noalloc(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype,
                                  void* stream, char* err, uint64_t cap) {
    if (M < 0 || N < 0 || K < 0) return sf::fail(SF_EINVAL, err, cap, "gemm_nn_noalloc: negative size");
    if (dtype != SF_DTYPE_F16 && dtype != SF_DTYPE_BF16)
        return sf::fail(SF_EINVAL, err, cap, "gemm_nn_noalloc: dtype %d is not fp16/bf16", dtype);
    if (M == 0 || N == 0) return SF_OK;
    if (!C || (K > 0 && (!A || !B))) return sf::fail(SF_EINVAL, err, cap, "gemm_nn_noalloc: null tensor pointer");
    cudaStream_t s = (cudaStream_t)stream;
    // B read in place, the general kernel, or K == 0: no scratch (no workspace in sf_gemm_nn).
    if (K == 0 || sf_gemm_nn_tc_supported(A, B, C, M, N, K)) return sf_gemm_nn_launch(A, B, C, M, N, K, dtype, 0, nullptr, 0, s, err, cap);
    // The tensor-core kernel on a transposed B: the array is 256-byte aligned, so only A, C and K
    // decide (A, already required to be aligned, stands in for the array in the predicate).
    if (!sf_gemm_nt_tc_supported(A, A, C, M, N, K)) return sf_gemm_nn_launch(A, B, C, M, N, K, dtype, 2, nullptr, 0, s, err, cap);
    const uint64_t need = (uint64_t)K * (uint64_t)N * 2u;
    if (need > kScratchBytes)
        return sf::fail(SF_EINVAL, err, cap,
                        "gemm_nn_noalloc: this shape needs B transposed (N %% 8 != 0 or B unaligned); K*N = %lld x %lld needs %llu bytes of transpose scratch and "
                        "the static scratch holds %llu bytes (use sf_gemm_nn with a caller workspace for larger problems)",
                        (long long)K, (long long)N, (unsigned long long)need, (unsigned long long)kScratchBytes);
    const int64_t gx = (N + 63) / 64, gy = (K + 63) / 64;
    if (gy > 65535) return sf::fail(SF_EINVAL, err, cap, "gemm_nn_noalloc: K=%lld too large for the transpose grid", (long long)K);
    void* scratch = nullptr;
    int rc = scratch_for_current_context(&scratch, err, cap);
    if (rc) return rc;
    noalloc_transpose16_kernel<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, s>>>((const uint16_t*)B, (uint16_t*)scratch, K, N);
    rc = sf::check_launch("gemm_nn_noalloc transpose launch", err, cap);
    if (rc) return rc;
    // The transposed B is [N, K]: the NT tensor-core product gives A . B.
    return sf_gemm_nt_tc_launch(A, scratch, C, M, N, K, dtype, false, s, err, cap);
}
