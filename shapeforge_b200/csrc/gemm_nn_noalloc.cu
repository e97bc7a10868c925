// sf_gemm_nn_noalloc: C[M,N] = A[M,K] . B[K,N] without any device allocation.
//
// Who needs this.  sf_gemm_nn runs the tensor-core kernel on a transposed copy of B, and that
// copy lives in a workspace the caller allocates.  Some callers cannot allocate device memory
// when they need the product:
//   * code enqueued from inside a host callback (cudaLaunchHostFunc), where CUDA API calls such
//     as cudaMalloc are not permitted at all;
//   * hosts whose device memory is entirely reserved up front by another allocator (a caching
//     allocator or a memory pool sized to the card): a raw cudaMalloc there fails or fragments
//     the pool;
//   * certified or real-time hosts that forbid dynamic allocation after start-up.
// For them this entry point keeps the transpose scratch in a fixed, file-scope device array.
//
// The price.  The array (SF_GEMM_NN_NOALLOC_MAX_SCRATCH_BYTES = 32 MiB) is reserved on every
// GPU that loads the library, for as long as the process lives.  Problems whose transposed B
// (K*N 16-bit elements) does not fit are rejected with SF_EINVAL.  All calls on a device share
// the one array, and it keeps whatever the previous call left there; nothing in it needs to
// start at zero, because every call overwrites the K*N elements it reads before reading them.
// Calls that overlap on the GPU (on different streams, or from several threads without
// ordering) race on the array and produce wrong results: serialise them on one stream.
//
// Set-up.  The first call on a device resolves the array's device address with
// cudaGetSymbolAddress while that device is current, and caches it.  Make that first call
// before any stream capture begins on the device.  In host code the array's name is only a
// host-side stand-in, never a device address, which is why the resolved pointer is what the
// kernels receive.
#include "sf_common.cuh"

#include <mutex>

// The transpose scratch shared by every call on a device (see above).
static __device__ __align__(256) uint8_t g_gemm_nn_scratch[SF_GEMM_NN_NOALLOC_MAX_SCRATCH_BYTES];

namespace {

constexpr uint64_t kScratchBytes = SF_GEMM_NN_NOALLOC_MAX_SCRATCH_BYTES;

std::mutex g_setup_mu;
void* g_scratch_ptr[64] = {nullptr};

// Resolve (once per device, with that device current) the device address of the scratch array.
int scratch_for_current_device(void** out, char* err, uint64_t cap) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return sf::fail(SF_EDEVICE, err, cap, "gemm_nn_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return sf::fail(SF_EDEVICE, err, cap, "gemm_nn_noalloc: device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_gemm_nn_scratch);
        if (e != cudaSuccess || !p)
            return sf::fail(SF_EDEVICE, err, cap, "gemm_nn_noalloc: cudaGetSymbolAddress of the scratch array failed: %s",
                            cudaGetErrorString(e));
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
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
    const uint64_t need = (uint64_t)K * (uint64_t)N * 2u;
    if (need > kScratchBytes)
        return sf::fail(SF_EINVAL, err, cap,
                        "gemm_nn_noalloc: K*N = %lld x %lld needs %llu bytes of transpose scratch; the static scratch holds %llu "
                        "bytes (use sf_gemm_nn with a caller workspace for larger problems)",
                        (long long)K, (long long)N, (unsigned long long)need, (unsigned long long)kScratchBytes);
    if (M == 0 || N == 0) return SF_OK;
    if (!C || (K > 0 && (!A || !B))) return sf::fail(SF_EINVAL, err, cap, "gemm_nn_noalloc: null tensor pointer");
    void* scratch = nullptr;
    int rc = scratch_for_current_device(&scratch, err, cap);
    if (rc) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    if (K > 0) {
        const int64_t gx = (N + 63) / 64, gy = (K + 63) / 64;
        if (gy > 65535) return sf::fail(SF_EINVAL, err, cap, "gemm_nn_noalloc: K=%lld too large for the transpose grid", (long long)K);
        noalloc_transpose16_kernel<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, s>>>((const uint16_t*)B, (uint16_t*)scratch, K, N);
        rc = sf::check_launch("gemm_nn_noalloc transpose launch", err, cap);
        if (rc) return rc;
    }
    // The transposed B is [N, K]: the NT product (tensor cores when the shape allows it, else the
    // general kernel) gives A . B.
    return sf_gemm_nt_launch(A, scratch, C, M, N, K, dtype, 0, s, err, cap);
}
