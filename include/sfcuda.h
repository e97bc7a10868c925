/*
 * sfcuda.h — C ABI of the ShapeForge B200 (sm_100a) execution backend.
 *
 * This is the native boundary the harness binds with ctypes (the B200 counterpart of the
 * reference's Metal batch encoder, tcenv/backends/metal/native_batch.m).  Every entry point
 * takes plain device pointers, sizes and a CUDA stream handle (cudaStream_t passed as void*),
 * never allocates or frees memory, and follows the native_batch.m status convention
 * (native_batch.m:43-46, :150, :191-194):
 *
 *     0  SF_OK       the work was enqueued (or completed, for calls that say so)
 *     2  SF_EINVAL   invalid arguments: nothing was launched
 *     3  SF_EDEVICE  the CUDA runtime reported an error
 *
 * On a non-zero status a NUL-terminated message is written into the caller-owned buffer
 * `err` of `cap` bytes (may be NULL / 0).  Launches are asynchronous on `stream`; only
 * sf_run_batch and sf_device_info synchronise.
 *
 * Tensor arguments are row-major and contiguous, in the ABI order of the task's OpSpec
 * `tensors` block (inputs, then outputs).  dtype codes are SF_DTYPE_*.
 */
#ifndef SFCUDA_H
#define SFCUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SF_API __attribute__((visibility("default")))
#else
#define SF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SF_OK 0
#define SF_EINVAL 2
#define SF_EDEVICE 3

#define SF_DTYPE_F16 0
#define SF_DTYPE_BF16 1
#define SF_DTYPE_F32 2
#define SF_DTYPE_I32 3

/* Library version string, e.g. "0.1.0+sm_100a". */
SF_API const char* sf_version(void);

/*
 * Device probe: replaces the Metal device probe behind Backend.probe
 * (tcenv/backends/base.py:223).  Synchronous.  `name` receives the device name.
 */
typedef struct sf_device_info {
    int32_t device;
    int32_t cc_major;
    int32_t cc_minor;
    int32_t sm_count;
    int64_t global_mem_bytes;
    int64_t l2_bytes;
    int32_t max_smem_per_block_optin;
    int32_t max_threads_per_block;
    int32_t clock_khz;
    int32_t mem_clock_khz;
    int32_t mem_bus_width_bits;
    char name[128];
} sf_device_info;

SF_API int sf_device_info_get(int32_t device, sf_device_info* out, char* err, uint64_t cap);

/*
 * Fill `nbytes` bytes at `dst` with the byte `value` (the guard 0xCD / poison 0xFF / zero
 * fills of tcenv/track/protocol.py:43-47, 107-143).  Asynchronous on `stream`.
 */
SF_API int sf_fill_bytes(void* dst, uint64_t nbytes, int32_t value, void* stream, char* err, uint64_t cap);

/*
 * Count the bytes in [ptr, ptr+nbytes) that differ from `value` into *count (device
 * uint64 counter, caller zeroes it).  Used to check guard bands and unwritten poison on the
 * device instead of copying whole buffers to the host.
 */
SF_API int sf_count_mismatch(const void* ptr, uint64_t nbytes, int32_t value, uint64_t* count_dev,
                      void* stream, char* err, uint64_t cap);

/* ---------------------------------------------------------------------------------------
 * Task operators.  Each replaces the candidate kernel dispatch of one OpSpec v2 task.
 * ------------------------------------------------------------------------------------- */

/*
 * rmsnorm: y[r,:] = x[r,:] * rsqrt(mean(x[r,:]^2) + eps) * w   (fp32 accumulation, one
 * rounding).  tasks/rmsnorm/reference.py:110-115, opspec.json:5.  x,y [rows, hidden], w [hidden].
 * dtype F16 or BF16.  rows >= 0, hidden >= 1.
 */
SF_API int sf_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t hidden, float eps,
               int32_t dtype, void* stream, char* err, uint64_t cap);

/*
 * silu: y = x * sigmoid(x) over n elements (tasks/silu/reference.py:105-108).
 * swiglu: y = gate * sigmoid(gate) * up (tasks/swiglu/reference.py:109-113).  F16 / BF16.
 */
SF_API int sf_silu(const void* x, void* y, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap);
SF_API int sf_swiglu(const void* gate, const void* up, void* y, int64_t n, int32_t dtype, void* stream, char* err,
               uint64_t cap);

/*
 * relu: y = max(x, 0), values <= 0 map to +0 and NaN propagates (tasks/relu/reference.py, reference()).
 * sigmoid: y = 1 / (1 + exp(-x)) (tasks/sigmoid/reference.py, reference()).
 * sigmoid_shift: y = sigmoid(x) + 1 (tasks/sigmoid_shift/reference.py, reference()).
 * fp32 arithmetic, one rounding to the F16 / BF16 output.
 */
SF_API int sf_relu(const void* x, void* y, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap);
SF_API int sf_sigmoid(const void* x, void* y, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap);
SF_API int sf_sigmoid_shift(const void* x, void* y, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap);

/*
 * lion: one Lion optimizer step over n elements (tasks/lion/reference.py, reference();
 * opspec.json formula): c = BETA1*m + (1-BETA1)*g, p_out = p*(1 - LR*WD) - LR*sign(c),
 * m_out = BETA2*m + (1-BETA2)*g.  Attribute domains LR > 0, WD >= 0, 0 < BETA1, BETA2 < 1
 * (SF_EINVAL otherwise).  F16 / BF16 tensors, fp32 arithmetic.
 */
SF_API int sf_lion(const void* p, const void* g, const void* m, void* p_out, void* m_out, int64_t n, double lr, double wd,
               double beta1, double beta2, int32_t dtype, void* stream, char* err, uint64_t cap);

/*
 * gemv: y[r] = sum_k A[r, k] * x[k], A [M, K] row-major, x [K], y [M] (tasks/gemv/reference.py,
 * reference()).  fp32 accumulation, F16 / BF16 storage; K == 0 writes +0.
 */
SF_API int sf_gemv(const void* A, const void* x, void* y, int64_t M, int64_t K, int32_t dtype, void* stream, char* err,
               uint64_t cap);

/*
 * softmax over the last axis of x [m, n] (tasks/softmax/reference.py:104-106) and
 * reduction_sum y[m] = sum_j x[m, j] (tasks/reduction_sum/reference.py:104-106); fp32
 * accumulation, F16 / BF16 storage.
 */
SF_API int sf_softmax(const void* x, void* y, int64_t m, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap);
SF_API int sf_reduction_sum(const void* x, void* y, int64_t m, int64_t n, int32_t dtype, void* stream, char* err,
               uint64_t cap);

/*
 * rope: rotate-half rotary embedding of x [B, H, S, D] with position = index along S and
 * inv_freq = base^(-i / (D/2)) (tasks/rope/reference.py:105-115).  D even.  F16 / BF16.
 */
SF_API int sf_rope(const void* x, void* y, int64_t B, int64_t H, int64_t S, int64_t D, double base, int32_t dtype,
               void* stream, char* err, uint64_t cap);

/*
 * bitdelta_gemm (tasks/bitdelta_gemm/reference.py:99-130): y[M,N] = scale * x[M,K] . W[K,N]
 * with W[k,n] = +1 if bit (k % 32) of bits[k/32, n] is set, else -1.  bits is [K/32, N] 32-bit
 * words; K % 32 == 0.  tcgen05 kernel with the signs expanded in shared memory.
 */
SF_API int sf_bitdelta_gemm(const void* x, const void* bits, void* y, int64_t M, int64_t N, int64_t K, float scale,
               int32_t dtype, void* stream, char* err, uint64_t cap);

/*
 * bitdelta_gemm_base (the 1-bit-delta fine-tune workload): y[M,N] = x[M,K] . (W_base[N,K] +
 * diag(alpha[N]) S[N,K])^T with S in {-1,+1} packed along K as s_words[N, K/32] (bit j of word
 * kb is column kb*32 + j, set = +1).  Swap-AB tcgen05 kernel, split-K over a cluster.
 */
SF_API int sf_bitdelta_gemm_base(const void* x, const void* w_base, const void* s_words, const void* alpha, void* y,
               int64_t M, int64_t N, int64_t K, int32_t dtype, void* stream, char* err, uint64_t cap);

/*
 * flash_attention forward: o = softmax(q . k^T * scale [+ causal mask]) . v over q, k, v, o
 * [B, H, S, D] (tasks/flash_attention/reference.py:113-119 with SM_SCALE = scale; causal != 0
 * keeps key j <= query i).  tcgen05 kernel for D in {64, 128}; general kernel otherwise (D <= 256).
 */
SF_API int sf_flash_attention(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t H, int64_t S,
               int64_t D, float scale, int32_t causal, int32_t dtype, void* stream, char* err, uint64_t cap);

/*
 * varlen_kda (tasks/varlen_kda/reference.py:323-374): packed-varlen Kimi Delta Attention forward.
 * q, k, v, g [T, H, D] and beta [T, H] in dtype; A_log [H], dt_bias [H*D], initial_state and
 * final_state [num_seqs, H, D, D] (V-first), scale [1] fp32; cu_seqlens [num_seqs + 1] int32
 * (negative entries = capacity sentinel: those sequences are skipped and left untouched).
 * lower_bound is the LOWER_BOUND attr.  D in {8, 16, 32, 64, 128}.
 */
SF_API int sf_varlen_kda(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
               const void* dt_bias, const void* initial_state, const void* cu_seqlens, const void* scale, void* output,
               void* final_state, int64_t num_seqs, int64_t H, int64_t D, float lower_bound, int32_t dtype, void* stream,
               char* err, uint64_t cap);

/*
 * varlen_kda with a caller workspace: the two-pass kernels (every 32-token chunk's operands,
 * norms and gates included, formed in parallel into `workspace`, then one state chain per
 * (sequence, head)) when D = 128 and `workspace` holds sf_varlen_kda_workspace_bytes(total_tokens,
 * num_seqs, H, D) bytes at a 256-byte-aligned address; otherwise as sf_varlen_kda.  total_tokens =
 * the rows of q (a sequence ending past it is reported through sf_kernel_status, code 2 where 96,
 * with no work done); the workspace needs no initialisation and may be reused once the call's work
 * on `stream` is done.  Replaces the same call as sf_varlen_kda (the task's kernel entry,
 * tasks/varlen_kda/reference.py:323-374); the reference's ABI has no workspace.
 */
SF_API uint64_t sf_varlen_kda_workspace_bytes(int64_t total_tokens, int64_t num_seqs, int64_t H, int64_t D);
SF_API int sf_varlen_kda_ws(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
               const void* dt_bias, const void* initial_state, const void* cu_seqlens, const void* scale, void* output,
               void* final_state, int64_t num_seqs, int64_t total_tokens, int64_t H, int64_t D, float lower_bound,
               int32_t dtype, void* workspace, uint64_t workspace_bytes, void* stream, char* err, uint64_t cap);

/*
 * kda: fixed-length Kimi Delta Attention forward (tasks/kda/reference.py reference(); opspec.json
 * formula): the varlen_kda recurrence over ONE sequence of N tokens, without cu_seqlens.
 * q, k, v, g [N, H, D] and beta [N, H] in dtype; A_log [H], dt_bias [H*D], scale [1] fp32;
 * initial_state and final_state [H, D, D] fp32 (V-first); lower_bound is the LOWER_BOUND attr.
 * The candidate-owned outputs of the task's host program: work_items [3, 2] u32 receives the
 * work list ((0, N) then two empty (N, 0) items), item_counts [1] i32 receives 1, and
 * handoff_states [2, H, D, D] fp32 (piece-boundary states) is not written, one piece having no
 * boundary.  D in {8, 16, 32, 64, 128}; work_items 4-byte aligned.
 */
SF_API int sf_kda(const void* q, const void* k, const void* v, const void* g, const void* beta, const void* a_log,
               const void* dt_bias, const void* initial_state, const void* scale, void* output, void* final_state,
               void* work_items, void* item_counts, void* handoff_states, int64_t N, int64_t H, int64_t D, float lower_bound,
               int32_t dtype, void* stream, char* err, uint64_t cap);

/*
 * varlen_kda_gated (the gated workload): same recurrence with q, k already L2-normalised, g the
 * fp32 log-decay [T, H, D] used directly, beta the fp32 gate [T, H] used directly, q times
 * `scale`, state starting at zero when initial_state is NULL.
 */
SF_API int sf_varlen_kda_gated(const void* q, const void* k, const void* v, const void* g, const void* beta,
               const void* cu_seqlens, const void* initial_state, void* output, void* final_state, int64_t num_seqs,
               int64_t H, int64_t D, float scale, int32_t dtype, void* stream, char* err, uint64_t cap);

/*
 * varlen_kda_gated with a caller workspace: the two-pass kernels (every 32-token chunk's operands
 * formed in parallel into `workspace`, then one state chain per (sequence, head)) when D = 128 and
 * `workspace` holds sf_varlen_kda_gated_workspace_bytes(total_tokens, num_seqs, H, D) bytes at a
 * 256-byte-aligned address; otherwise as sf_varlen_kda_gated.  total_tokens = cu_seqlens[num_seqs]
 * (the rows of q); the workspace needs no initialisation and may be reused once the call's work on
 * `stream` is done.  No reference counterpart: the reference's varlen_kda ABI has no workspace.
 */
SF_API uint64_t sf_varlen_kda_gated_workspace_bytes(int64_t total_tokens, int64_t num_seqs, int64_t H, int64_t D);
SF_API int sf_varlen_kda_gated_ws(const void* q, const void* k, const void* v, const void* g, const void* beta,
               const void* cu_seqlens, const void* initial_state, void* output, void* final_state, int64_t num_seqs,
               int64_t total_tokens, int64_t H, int64_t D, float scale, int32_t dtype, void* workspace,
               uint64_t workspace_bytes, void* stream, char* err, uint64_t cap);

/*
 * mamba2_chunk_scan (tasks/mamba2_chunk_scan/reference.py:106-127): the Mamba-2 SSD chunk scan of
 * one B/C group.  x [B,L,H,P], dt [B,L,H], dA_cumsum [B,H,NC,chunk] (NC = L / chunk),
 * Bmat/Cmat [B,L,N], Dskip [H], states [B,NC,H,P,N] in, y [B,L,H,P] out, all in dtype, fp32
 * arithmetic, one rounding of y.  tcgen05 kernel when chunk = P = N = 64 and x, Bmat, Cmat,
 * states, y are 16-byte aligned; general fp32 kernel otherwise.  L must be a multiple of chunk.
 */
SF_API int sf_mamba2_chunk_scan(const void* x, const void* dt, const void* dA_cumsum, const void* Bmat, const void* Cmat,
               const void* Dskip, const void* states, void* y, int64_t B, int64_t L, int64_t H, int64_t P, int64_t N,
               int64_t chunk, int32_t dtype, void* stream, char* err, uint64_t cap);

/*
 * gemm_nt: C[M,N] = A[M,K] . B[N,K]^T, fp16 or bf16 in, fp32 accumulation, one rounding
 * (the dense-gemm workload; the oracle is tasks/gemm/reference.py:110-114 applied to B^T).
 * tcgen05/TMEM/TMA kernel when the bases are 16-byte aligned and K % 8 == 0, else the general
 * fallback kernel.  Any M, N, K >= 0 (K == 0 writes zeros).
 */
SF_API int sf_gemm_nt(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype,
               void* stream, char* err, uint64_t cap);

/*
 * gemm_nn: C[M,N] = A[M,K] . B[K,N] — the tasks/gemm contract (reference.py:110-114,
 * opspec.json:5: B row-major [K,N]).  With 16-byte aligned tensors, K % 8 == 0 and N % 8 == 0 the
 * tensor-core kernel reads B in place (sf_gemm_nn_workspace_bytes returns 0).  Otherwise, with a
 * workspace of at least sf_gemm_nn_workspace_bytes(M,N,K,dtype) bytes (16-byte aligned,
 * caller-owned) B is transposed into it and the tensor-core kernel runs; with workspace == NULL
 * the general fallback kernel runs.
 */
SF_API uint64_t sf_gemm_nn_workspace_bytes(int64_t M, int64_t N, int64_t K, int32_t dtype);
SF_API int sf_gemm_nn(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype,
               void* workspace, uint64_t workspace_bytes, void* stream, char* err, uint64_t cap);

/*
 * gemm_silu: C[M,N] = silu(A[M,K] . B[K,N]), silu(v) = v * sigmoid(v) on the fp32 product
 * (tasks/gemm_silu/reference.py, reference(); opspec.json formula).  Same layouts, dispatch and
 * workspace rule as sf_gemm_nn (sf_gemm_nn_workspace_bytes sizes it); the SiLU is the epilogue
 * of whichever kernel runs.
 */
SF_API int sf_gemm_silu(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype,
               void* workspace, uint64_t workspace_bytes, void* stream, char* err, uint64_t cap);

/*
 * gemm_nn without any device allocation (no counterpart in the reference).  Same result as
 * sf_gemm_nn with a workspace, for callers that cannot allocate device memory at call time:
 * hosts whose device memory is fully reserved by another allocator they give no access to, and
 * certified/real-time hosts that forbid allocation after start-up.  Shapes sf_gemm_nn runs
 * without a workspace (N % 8 == 0 with aligned tensors, the general kernel, K == 0) run the same
 * way here and have no size limit.  Shapes that need B transposed use a fixed file-scope device
 * array of SF_GEMM_NN_NOALLOC_MAX_SCRATCH_BYTES, held on every GPU that loads the library until
 * exit; those with K*N*2 bytes above it are rejected with SF_EINVAL.  The first such call in a
 * CUDA context resolves the array's address (cudaGetSymbolAddress) — make it before any stream
 * capture.  All calls share the array: calls that overlap on the GPU race; serialise them on
 * one stream.  Like every entry point here it makes CUDA API calls, so it must not be called
 * from a host function or stream callback.
 */
#define SF_GEMM_NN_NOALLOC_MAX_SCRATCH_BYTES (32ull * 1024ull * 1024ull)
SF_API int sf_gemm_nn_noalloc(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype,
               void* stream, char* err, uint64_t cap);

/*
 * Read and clear the sticky status word of the tcgen05 kernels: code 0 = ok, 1 = a bounded
 * pipeline wait gave up (the launch's output is invalid); `where` names the wait.  Synchronises
 * `stream`.  Replaces the reference's launch watchdog verdict for device-side stalls
 * (tcenv/evaluate.py:1029-1051) without trapping the GPU.
 */
SF_API int sf_kernel_status(uint32_t* code, uint32_t* where, void* stream, char* err, uint64_t cap);

/* ---------------------------------------------------------------------------------------
 * Compiled candidate kernels (the Candidate/Harness split).  The harness compiles a candidate
 * CUDA source to an sm_100a cubin, loads it here and launches its kernels; replaces the Metal
 * pipeline creation and dispatch (tcenv/backends/metal/runtime.py:306, :593).
 * ------------------------------------------------------------------------------------- */

/* Load a cubin/fatbin image; *module receives an opaque handle (cudaLibrary_t). */
SF_API int sf_module_load(const void* image, uint64_t size, void** module, char* err, uint64_t cap);
SF_API int sf_module_unload(void* module, char* err, uint64_t cap);
/* Resolve an extern "C" kernel by name; *function receives an opaque handle (cudaKernel_t). */
SF_API int sf_module_get_function(void* module, const char* name, void** function, char* err, uint64_t cap);
/* Launch `function` with cudaLaunchKernel semantics: args[i] points at the i-th parameter's value. */
SF_API int sf_launch_kernel(void* function, uint32_t gx, uint32_t gy, uint32_t gz, uint32_t bx, uint32_t by, uint32_t bz,
               uint32_t smem, void* stream, void** args, char* err, uint64_t cap);

/* ---------------------------------------------------------------------------------------
 * Generic dispatch + timed batches (the taic_metal_run_batch replacement).
 * ------------------------------------------------------------------------------------- */

#define SF_OP_RMSNORM 1
#define SF_OP_GEMM_NT 2
#define SF_OP_GEMM_NN 3
#define SF_OP_SILU 4
#define SF_OP_SWIGLU 5
#define SF_OP_SOFTMAX 6
#define SF_OP_REDUCTION_SUM 7
#define SF_OP_ROPE 8
#define SF_OP_BITDELTA 9
#define SF_OP_BITDELTA_BASE 10
#define SF_OP_ATTENTION 11
#define SF_OP_KDA 12
#define SF_OP_KDA_GATED 13
#define SF_OP_MAMBA2 14
#define SF_OP_RELU 15
#define SF_OP_SIGMOID 16
#define SF_OP_SIGMOID_SHIFT 17
#define SF_OP_LION 18
#define SF_OP_GEMV 19
#define SF_OP_GEMM_SILU 20
#define SF_OP_KDA_FIXED 21

typedef struct sf_op_desc {
    int32_t op;       /* SF_OP_* */
    int32_t dtype;    /* SF_DTYPE_* of the task's type variable T */
    int32_t variant;  /* 0 = default dispatch; op-specific forced variant otherwise */
    int32_t flags;    /* op-specific (e.g. causal) */
    int64_t dims[8];  /* op-specific sizes, see sf_run_op */
    double attrs[4];  /* op-specific scalar attributes (eps, scale, ...) */
} sf_op_desc;

/* Number of tensor arguments op `op` takes (0 for an unknown op). */
SF_API int32_t sf_op_nargs(int32_t op);

/*
 * Enqueue one launch of `desc` with tensor pointers `args` (sf_op_nargs(desc->op) entries,
 * ABI order).  dims/attrs per op:
 *   SF_OP_RMSNORM   dims = {rows, hidden}          attrs = {eps}       args = {x, w, y}
 *   SF_OP_GEMM_NT   dims = {M, N, K}                                   args = {A, B, C}
 *   SF_OP_GEMM_NN   dims = {M, N, K, ws_bytes}                         args = {A, B, C, ws}
 *   SF_OP_SILU      dims = {n}                                         args = {x, y}
 *   SF_OP_SWIGLU    dims = {n}                                         args = {gate, up, y}
 *   SF_OP_SOFTMAX   dims = {m, n}                                      args = {x, y}
 *   SF_OP_REDUCTION_SUM dims = {m, n}                                  args = {x, y}
 *   SF_OP_ROPE      dims = {B, H, S, D}            attrs = {base}      args = {x, y}
 *   SF_OP_BITDELTA  dims = {M, N, K}               attrs = {scale}     args = {x, bits, y}
 *   SF_OP_BITDELTA_BASE dims = {M, N, K}                               args = {x, w_base, s_words, alpha, y}
 *   SF_OP_ATTENTION dims = {B, H, S, D}  attrs = {scale}  flags bit 0 = causal  args = {q, k, v, o}
 *   SF_OP_KDA       dims = {num_seqs, H, D, total_tokens, ws_bytes}  attrs = {lower_bound}
 *                   args = {q, k, v, g, beta, A_log, dt_bias, initial_state, cu_seqlens, scale, output, final_state,
 *                           workspace (may be NULL: the 16-token chunked kernel)}
 *                   variant 4 forces the two-pass kernels, 1 the 16-token chunked kernel, 2 the recurrent one
 *   SF_OP_KDA_GATED dims = {num_seqs, H, D, total_tokens, ws_bytes}  attrs = {scale}
 *                   args = {q, k, v, g, beta, cu_seqlens, initial_state (may be NULL), output, final_state,
 *                           workspace (may be NULL: single-pass kernels)}
 *                   variant 4 forces the two-pass kernels, 1 the single-pass 32-token kernel
 *   SF_OP_MAMBA2    dims = {B, L, H, P, N, chunk}
 *                   args = {x, dt, dA_cumsum, Bmat, Cmat, Dskip, states, y}
 *   SF_OP_RELU / SF_OP_SIGMOID / SF_OP_SIGMOID_SHIFT  dims = {n}       args = {x, y}
 *   SF_OP_LION      dims = {n}   attrs = {LR, WD, BETA1, BETA2}        args = {p, g, m, p_out, m_out}
 *   SF_OP_GEMV      dims = {M, K}                                      args = {A, x, y}
 *   SF_OP_GEMM_SILU dims = {M, N, K, ws_bytes}                         args = {A, B, C, ws}
 *   SF_OP_KDA_FIXED dims = {N, H, D}  attrs = {lower_bound}
 *                   args = {q, k, v, g, beta, A_log, dt_bias, initial_state, scale, output, final_state,
 *                           work_items, item_counts, handoff_states}
 * desc->variant: 0 = exact dispatch with fallback, 1 = force the specialised (tensor-core /
 * vectorised) kernel, 2 = force the general fallback kernel.
 */
SF_API int sf_run_op(const sf_op_desc* desc, const void* const* args, uint64_t nargs, void* stream,
              char* err, uint64_t cap);

/*
 * Timed batch (mirror of taic_metal_run_batch, native_batch.m:128): enqueue `iters`
 * launches of `desc`, launch i binding argument set (i % nsets) from `args`
 * ([nsets][nargs] flattened), bracketed by two CUDA events on `stream`; synchronise and
 * write the elapsed device seconds to *gpu_s.  With use_graph != 0 the `iters` launches are
 * captured once into a CUDA graph (outside the timed region) and the graph launch is timed,
 * which removes per-launch CPU overhead for launch-bound shards.
 */
SF_API int sf_run_batch(const sf_op_desc* desc, const void* const* args, uint64_t nargs, uint64_t nsets,
                 uint64_t iters, int32_t use_graph, void* stream, double* gpu_s, char* err,
                 uint64_t cap);

#ifdef __cplusplus
}
#endif

#endif /* SFCUDA_H */
