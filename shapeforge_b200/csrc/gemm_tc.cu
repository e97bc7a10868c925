// Dense GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//   C[M,N] = A[M,K] . B[N,K]^T      (both operands K-major; fp16 or bf16 in, fp32 accumulate,
//                                    one rounding to the input dtype at the output)
//
// This is the gemm_nt workload (dense gemm, C = A.B^T).  The reference task tasks/gemm stores B as
// [K, N]; the same kernel reads that layout directly as an MN-major B operand (BMN = true): each
// K-block of B arrives as 64 x 64 TMA boxes (64 N columns of 128 bytes for 64 K rows) and the
// MMA's B descriptor walks 16 K rows (2 KB) per instruction with 8 KB between 64-column blocks.
// With SILU = true the epilogue stores silu(acc) = acc * sigmoid(acc) instead: the gemm_silu task
// (tasks/gemm_silu/reference.py), fused at no extra memory traffic.
//
// Persistent, warp-specialised kernel, one CTA per SM (192 KB of pipeline shared memory):
//   warp 0      TMA producer: 128x64 A box + 256x64 B box per K-block, 128-byte swizzle,
//               into a 4-stage ring of shared memory guarded by full/empty mbarriers;
//   warp 1      MMA issuer: one thread issues 4 x tcgen05.mma (M=128, N=256, K=16) per
//               K-block into a TMEM accumulator, tcgen05.commit releases the smem stage;
//   warps 2..5  epilogue: tcgen05.ld of the 128x256 fp32 accumulator (each warp its 32-lane
//               TMEM quadrant), convert, 16-byte stores to C.
// The TMEM accumulator is double-buffered (2 x 256 columns), so the epilogue of tile i
// overlaps the main loop of tile i+1.  Work units are visited round-robin by the persistent
// CTAs; when the tiles left after the last full round fit twice on the SMs, each of them is split
// into two 128-column halves (N=128 MMAs), so the last round takes half a tile instead of a whole
// one (4096^3: 3.5 instead of 4 tile times per CTA).  Every mbarrier wait is bounded (sm100::mbar_wait):
// a wait that gives up records a status word and the CTA drains to its teardown.
//
// Small problems (K-major B, at most one SM's worth of 128 x 64 tiles) take gemm_nt_small_kernel
// instead: one CTA per 128 x 64 tile, an 8-stage ring of 64-deep K-blocks (24 KB each), so up to
// K = 512 every load of the CTA is in flight at once and the tile costs one memory round trip; the
// persistent kernel would leave most SMs idle and stream its K-blocks through two ring rounds.
#include "sf_common.cuh"
#include "sm100.cuh"
#include "tma_host.cuh"

#include <cudaTypedefs.h>
#include <algorithm>
#include <mutex>
#include <type_traits>

// Status word of the tcgen05 kernels in this file: a bounded wait that gave up records where.
// Sticky until read by sf_gemm_status_read (a module global: the library allocates nothing).
__device__ sm100::KernelStatus g_gemm_status;

namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;  // 64 x 16-bit = 128 bytes: one swizzle row
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = NUM_ACC * BN;  // 512
constexpr int NUM_THREADS = 192;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*alignment slack*/ + 256 /*barriers*/;

struct __align__(8) Barriers {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t acc_full[NUM_ACC];
    uint64_t acc_empty[NUM_ACC];
    uint32_t tmem_base;
};

// Grouped rasterisation: tiles are visited in column-major groups of GROUP_M tile rows so
// concurrently running CTAs share A and B panels in L2.
constexpr int GROUP_M = 16;

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
    const int per_group = GROUP_M * tiles_n;
    const int group = tile / per_group;
    const int first_m = group * GROUP_M;
    const int rows = min(tiles_m - first_m, GROUP_M);
    const int in_group = tile - group * per_group;
    tm = first_m + in_group % rows;
    tn = in_group / rows;
}

// Work unit u: a full 128 x 256 tile for u < full_units, else half `half` (0/1, 128 columns each)
// of tile full_units + (u - full_units) / 2.
__device__ __forceinline__ void unit_coords(int u, int full_units, int tiles_m, int tiles_n, int& tm, int& tn, int& half) {
    if (u < full_units) {
        tile_coords(u, tiles_m, tiles_n, tm, tn);
        half = -1;
    } else {
        const int h = u - full_units;
        tile_coords(full_units + (h >> 1), tiles_m, tiles_n, tm, tn);
        half = h & 1;
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

template <typename T, bool BMN, bool SILU>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_nt_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_bh, T* __restrict__ C, int M, int N, int K, int full_units,
                      int total_units, sm100::KernelStatus* status) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle atoms.
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Barriers* bars = reinterpret_cast<Barriers*>(smem + STAGES * STAGE_BYTES);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tiles_m = (M + BM - 1) / BM;
    const int tiles_n = (N + BN - 1) / BN;
    const int num_kb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            sm100::mbar_init(&bars->full[s], 1);
            sm100::mbar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < NUM_ACC; ++a) {
            sm100::mbar_init(&bars->acc_full[a], 1);
            sm100::mbar_init(&bars->acc_empty[a], 4 * 32);
        }
        sm100::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        sm100::tma_prefetch_desc(&tmap_a);
        sm100::tma_prefetch_desc(&tmap_b);
        sm100::tma_prefetch_desc(&tmap_bh);
    }
    if (warp == 1) {
        sm100::tmem_alloc(&bars->tmem_base, TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
                int tm, tn, half;
                unit_coords(u, full_units, tiles_m, tiles_n, tm, tn, half);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!sm100::mbar_wait(&bars->empty[stage], phase ^ 1u, status, 1)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + stage * STAGE_BYTES;
                    uint8_t* sb = sa + A_BYTES;
                    sm100::mbar_arrive_expect_tx(&bars->full[stage], half < 0 ? STAGE_BYTES : A_BYTES + B_BYTES / 2);
                    sm100::tma_load_2d(sa, &tmap_a, &bars->full[stage], kb * BK, tm * BM);
                    if (BMN) {
                        // B [K, N]: 64-column boxes of 64 K rows (8 KB each), N-block nb at sb + 8 KB * nb.
                        const int n0 = tn * BN + (half < 0 ? 0 : half * (BN / 2));
                        const int nblocks = half < 0 ? BN / 64 : BN / 128;
                        for (int nb = 0; nb < nblocks; ++nb)
                            sm100::tma_load_2d(sb + nb * (64 * BK * 2), &tmap_b, &bars->full[stage], n0 + nb * 64, kb * BK);
                    } else if (half < 0) {
                        sm100::tma_load_2d(sb, &tmap_b, &bars->full[stage], kb * BK, tn * BN);
                    } else {
                        sm100::tma_load_2d(sb, &tmap_bh, &bars->full[stage], kb * BK, tn * BN + half * (BN / 2));
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Drain: wait (bounded) until the MMA warp has released every stage, so no TMA
            // write into shared memory is still in flight at teardown.
            for (int s = 0; s < STAGES && ok; ++s) {
                if (!sm100::mbar_wait(&bars->empty[stage], phase ^ 1u, status, 2)) break;
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
            constexpr uint32_t idesc_full = BMN ? sm100::idesc_f16_bmn(BM, BN, BF) : sm100::idesc_f16(BM, BN, BF);
            constexpr uint32_t idesc_half = BMN ? sm100::idesc_f16_bmn(BM, BN / 2, BF) : sm100::idesc_f16(BM, BN / 2, BF);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
                const uint32_t idesc = u < full_units ? idesc_full : idesc_half;
                if (!sm100::mbar_wait(&bars->acc_empty[acc], acc_phase ^ 1u, status, 3)) break;
                sm100::tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!sm100::mbar_wait(&bars->full[stage], phase, status, 4)) {
                        ok = false;
                        break;
                    }
                    sm100::tc_fence_after();
                    const uint32_t sa = sm100::smem_u32(smem + stage * STAGE_BYTES);
                    const uint32_t sb = sa + A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        const uint64_t ad = sm100::smem_desc_k_sw128(sa + k * 32);
                        const uint64_t bd = BMN ? sm100::smem_desc_mn_sw128(sb + (uint32_t)(k * 16 * 128), 64 * BK * 2, 1024)
                                                : sm100::smem_desc_k_sw128(sb + k * 32);
                        sm100::mma_f16(d_tmem, ad, bd, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    }
                    sm100::mma_commit(&bars->empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                sm100::mma_commit(&bars->acc_full[acc]);
                if (++acc == NUM_ACC) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quad = warp & 3;  // TMEM lane quadrant this warp may access
        const int row_in_tile = quad * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        const bool vec_ok = (N % 8) == 0;
        for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
            int tm, tn, half;
            unit_coords(u, full_units, tiles_m, tiles_n, tm, tn, half);
            const int width = half < 0 ? BN : BN / 2;
            const int col_base = tn * BN + (half < 0 ? 0 : half * (BN / 2));
            if (!sm100::mbar_wait(&bars->acc_full[acc], acc_phase, status, 5)) break;
            sm100::tc_fence_after();
            const int row = tm * BM + row_in_tile;
            const uint32_t t_base = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
            for (int c = 0; c < width; c += 32) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(t_base + (uint32_t)c, r);
                sm100::tmem_ld_wait();
                // gemm_silu: v * sigmoid(v) in fp32 on the accumulator (tasks/gemm_silu/reference.py
                // applies it to the fp32 product; v = -inf gives -inf * 0 = NaN as there).  The
                // branch-free packed sigmoid keeps the 32 values of one TMEM load independent.
                if (SILU) {
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        const float2 v = make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
                        const float2 o = sf::f2_mul(v, sf::sigmoid2_nr(v));
                        r[j] = __float_as_uint(o.x);
                        r[j + 1] = __float_as_uint(o.y);
                    }
                }
                const int col0 = col_base + c;
                if (row < M) {
                    T* dst = C + (size_t)row * (size_t)N + col0;
                    if (vec_ok && col0 + 32 <= N) {
                        uint32_t p[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) p[j] = pack2<T>(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                        for (int j = 0; j < 4; ++j) d4[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (col0 + j < N) dst[j] = sf::Dt<T>::from_f(__uint_as_float(r[j]));
                        }
                    }
                }
            }
            sm100::tc_fence_before();
            sm100::mbar_arrive(&bars->acc_empty[acc]);
            if (++acc == NUM_ACC) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
    }

    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 1) sm100::tmem_dealloc(tmem_base, TMEM_COLS);
}

// ---- small problems: one 128 x 64 tile per CTA, all K-blocks in flight ---------------------------
constexpr int SBN = 64;
constexpr int S_STAGES = 8;
constexpr int S_B_BYTES = SBN * BK * 2;  // 8 KB
constexpr int S_STAGE_BYTES = A_BYTES + S_B_BYTES;
constexpr int S_TMEM_COLS = SBN;
constexpr int S_SMEM_BYTES = S_STAGES * S_STAGE_BYTES + 1024 + 256;

struct __align__(8) SmallBarriers {
    uint64_t full[S_STAGES];
    uint64_t empty[S_STAGES];
    uint64_t acc_full;
    uint32_t tmem_base;
};

template <typename T, bool SILU>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_nt_small_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, T* __restrict__ C, int M,
                         int N, int K, sm100::KernelStatus* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    SmallBarriers* bars = reinterpret_cast<SmallBarriers*>(smem + S_STAGES * S_STAGE_BYTES);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tiles_n = (N + SBN - 1) / SBN;
    const int tm = blockIdx.x / tiles_n, tn = blockIdx.x - tm * tiles_n;  // neighbouring CTAs share A rows
    const int num_kb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S_STAGES; ++s) {
            sm100::mbar_init(&bars->full[s], 1);
            sm100::mbar_init(&bars->empty[s], 1);
        }
        sm100::mbar_init(&bars->acc_full, 1);
        sm100::fence_mbar_init();
    }
    if (warp == 1) {
        sm100::tmem_alloc(&bars->tmem_base, S_TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < num_kb; ++kb) {
                const int stage = kb % S_STAGES;
                // Reuse of a stage (K > 512) waits for the MMAs that read it; the first round passes.
                if (!sm100::mbar_wait(&bars->empty[stage], ((uint32_t)(kb / S_STAGES) & 1u) ^ 1u, status, 11)) break;
                uint8_t* sa = smem + stage * S_STAGE_BYTES;
                sm100::mbar_arrive_expect_tx(&bars->full[stage], S_STAGE_BYTES);
                sm100::tma_load_2d(sa, &tmap_a, &bars->full[stage], kb * BK, tm * BM);
                sm100::tma_load_2d(sa + A_BYTES, &tmap_b, &bars->full[stage], kb * BK, tn * SBN);
                issued = kb + 1;
            }
            // Drain: the last ring of loads has landed (bounded), so no TMA write into shared memory
            // is in flight at teardown even if a wait elsewhere gave up.
            for (int kb = max(0, issued - S_STAGES); kb < issued; ++kb)
                if (!sm100::mbar_wait(&bars->full[kb % S_STAGES], (uint32_t)(kb / S_STAGES) & 1u, status, 14)) break;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;
            constexpr uint32_t idesc = sm100::idesc_f16(BM, SBN, BF);
            bool ok = true;
            for (int kb = 0; kb < num_kb; ++kb) {
                const int stage = kb % S_STAGES;
                if (!sm100::mbar_wait(&bars->full[stage], (uint32_t)(kb / S_STAGES) & 1u, status, 12)) {
                    ok = false;
                    break;
                }
                sm100::tc_fence_after();
                const uint32_t sa = sm100::smem_u32(smem + stage * S_STAGE_BYTES);
                const uint32_t sb = sa + A_BYTES;
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)
                    sm100::mma_f16(tmem_base, sm100::smem_desc_k_sw128(sa + k * 32), sm100::smem_desc_k_sw128(sb + k * 32), idesc,
                                   (kb > 0 || k > 0) ? 1u : 0u);
                sm100::mma_commit(&bars->empty[stage]);
            }
            if (ok) sm100::mma_commit(&bars->acc_full);
        }
    } else {
        const int quad = warp & 3;
        const int row = tm * BM + quad * 32 + lane;
        const bool vec_ok = (N % 8) == 0;
        if (sm100::mbar_wait(&bars->acc_full, 0, status, 13)) {
            sm100::tc_fence_after();
            const uint32_t t_base = tmem_base + ((uint32_t)(quad * 32) << 16);
#pragma unroll 1
            for (int c = 0; c < SBN; c += 32) {
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(t_base + (uint32_t)c, r);
                sm100::tmem_ld_wait();
                if (SILU) {
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        const float2 v = make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
                        const float2 o = sf::f2_mul(v, sf::sigmoid2_nr(v));
                        r[j] = __float_as_uint(o.x);
                        r[j + 1] = __float_as_uint(o.y);
                    }
                }
                const int col0 = tn * SBN + c;
                if (row < M) {
                    T* dst = C + (size_t)row * (size_t)N + col0;
                    if (vec_ok && col0 + 32 <= N) {
                        uint32_t p[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) p[j] = pack2<T>(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                        for (int j = 0; j < 4; ++j) d4[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (col0 + j < N) dst[j] = sf::Dt<T>::from_f(__uint_as_float(r[j]));
                        }
                    }
                }
            }
        }
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    if (warp == 1) sm100::tmem_dealloc(tmem_base, S_TMEM_COLS);
}

// ---- host side ----------------------------------------------------------------------------------

template <typename T, bool BMN, bool SILU>
int launch_tc(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, cudaStream_t stream, char* err,
              uint64_t cap) {
    const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    CUtensorMap ma, mb, mbh;
    int rc = sf::tmap_kmajor(&ma, A, M, K, BM, bf16, err, cap);
    if (rc) return rc;
    if (BMN) {
        // B [K, N] row-major: 64-element (128-byte) inner boxes along N, 64 K rows.
        rc = sf::tmap_kmajor(&mb, B, K, N, BK, bf16, err, cap);
        mbh = mb;
    } else {
        rc = sf::tmap_kmajor(&mb, B, N, K, BN, bf16, err, cap);
        if (!rc) rc = sf::tmap_kmajor(&mbh, B, N, K, BN / 2, bf16, err, cap);
    }
    if (rc) return rc;
    int dev = 0;
    cudaGetDevice(&dev);
    sm100::KernelStatus* st = nullptr;
    if (cudaGetSymbolAddress((void**)&st, g_gemm_status) != cudaSuccess || !st)
        return sf::fail(SF_EDEVICE, err, cap, "gemm: cannot resolve the status word");
    const int64_t sms = std::max(1, sf::sm_count());
    const int64_t small_ctas = ((M + BM - 1) / BM) * ((N + SBN - 1) / SBN);
    if (!BMN && small_ctas <= sms) {
        // At most one 128 x 64 tile per SM: the small-problem kernel.
        CUtensorMap mb64;
        rc = sf::tmap_kmajor(&mb64, B, N, K, SBN, bf16, err, cap);
        if (rc) return rc;
        static std::atomic<uint64_t> small_attr_done{0};
        if (sf::once_per_device(small_attr_done))
            cudaFuncSetAttribute(gemm_nt_small_kernel<T, SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, S_SMEM_BYTES);
        gemm_nt_small_kernel<T, SILU><<<(unsigned)small_ctas, NUM_THREADS, S_SMEM_BYTES, stream>>>(ma, mb64, (T*)C, (int)M, (int)N,
                                                                                               (int)K, st);
        return sf::check_launch("gemm_nt small tcgen05 launch", err, cap);
    }
    static std::atomic<uint64_t> attr_done{0};
    if (sf::once_per_device(attr_done))
        cudaFuncSetAttribute(gemm_nt_tc_kernel<T, BMN, SILU>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    // Tiles left over after the last full round of the persistent CTAs are split into halves when
    // the halves still fit in one round.
    const int64_t rounds = tiles / sms, tail = tiles - rounds * sms;
    int64_t full_units = tiles, total_units = tiles;
    if (tail > 0 && 2 * tail <= sms) {
        full_units = rounds * sms;
        total_units = full_units + 2 * tail;
    }
    if (total_units > 0x7fffffffLL) return sf::fail(SF_EINVAL, err, cap, "gemm: too many tiles");
    const int grid = (int)std::min<int64_t>(total_units, sms);
    gemm_nt_tc_kernel<T, BMN, SILU><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(ma, mb, mbh, (T*)C, (int)M, (int)N, (int)K, (int)full_units,
                                                                         (int)total_units, st);
    return sf::check_launch("gemm_nt tcgen05 launch", err, cap);
}

}  // namespace

// True when the tcgen05/TMA path can run this problem: 16-byte aligned bases, K % 8 == 0 (TMA
// row strides are multiples of 16 bytes) and sizes within the 32-bit coordinate range.
bool sf_gemm_nt_tc_supported(const void* A, const void* B, const void* C, int64_t M, int64_t N, int64_t K) {
    return sf::aligned16(A) && sf::aligned16(B) && sf::aligned16(C) && (K % 8) == 0 && M > 0 && N > 0 && K > 0 &&
           M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31);
}

// silu = true applies the gemm_silu epilogue to the accumulator before the store.
int sf_gemm_nt_tc_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, bool silu,
                         cudaStream_t stream, char* err, uint64_t cap) {
    if (dtype == SF_DTYPE_F16)
        return silu ? launch_tc<__half, false, true>(A, B, C, M, N, K, stream, err, cap)
                    : launch_tc<__half, false, false>(A, B, C, M, N, K, stream, err, cap);
    if (dtype == SF_DTYPE_BF16)
        return silu ? launch_tc<__nv_bfloat16, false, true>(A, B, C, M, N, K, stream, err, cap)
                    : launch_tc<__nv_bfloat16, false, false>(A, B, C, M, N, K, stream, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "gemm: dtype %d is not fp16/bf16", dtype);
}

// C = A . B with B stored [K, N], read as an MN-major operand: additionally needs N % 8 == 0 (B's
// rows are TMA strides, multiples of 16 bytes).
bool sf_gemm_nn_tc_supported(const void* A, const void* B, const void* C, int64_t M, int64_t N, int64_t K) {
    return sf_gemm_nt_tc_supported(A, B, C, M, N, K) && (N % 8) == 0;
}

int sf_gemm_nn_tc_launch(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int32_t dtype, bool silu,
                         cudaStream_t stream, char* err, uint64_t cap) {
    if (dtype == SF_DTYPE_F16)
        return silu ? launch_tc<__half, true, true>(A, B, C, M, N, K, stream, err, cap)
                    : launch_tc<__half, true, false>(A, B, C, M, N, K, stream, err, cap);
    if (dtype == SF_DTYPE_BF16)
        return silu ? launch_tc<__nv_bfloat16, true, true>(A, B, C, M, N, K, stream, err, cap)
                    : launch_tc<__nv_bfloat16, true, false>(A, B, C, M, N, K, stream, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "gemm: dtype %d is not fp16/bf16", dtype);
}

// Read (and clear) the device status word of the tcgen05 kernels on the current device.
int sf_gemm_status_read(uint32_t* code, uint32_t* where, cudaStream_t stream) {
    sm100::KernelStatus h{0, 0};
    if (cudaMemcpyFromSymbolAsync(&h, g_gemm_status, sizeof(h), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
        return SF_EDEVICE;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return SF_EDEVICE;
    if (h.code) {
        const sm100::KernelStatus zero{0, 0};
        cudaMemcpyToSymbolAsync(g_gemm_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream);
        cudaStreamSynchronize(stream);
    }
    *code = h.code;
    *where = h.where;
    return SF_OK;
}
