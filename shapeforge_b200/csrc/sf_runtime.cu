// Runtime half of the C ABI: device probe, byte fills and checks, generic op dispatch and the
// timed batch runner (the B200 replacement of the Metal batch encoder,
// tcenv/backends/metal/native_batch.m:128 taic_metal_run_batch).
#include "sf_common.cuh"

#include <vector>

namespace sf {

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (cached[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

}  // namespace sf

namespace {

__global__ void fill_bytes_kernel(uint8_t* __restrict__ dst, uint64_t n, uint8_t value) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    // Head up to 16-byte alignment, then 16-byte stores, then the tail.
    const uint64_t head = (16 - (reinterpret_cast<uintptr_t>(dst) & 15)) & 15;
    const uint64_t h = head < n ? head : n;
    if (i < h) dst[i] = value;
    const uint64_t nvec = (n - h) / 16;
    uint4* v = reinterpret_cast<uint4*>(dst + h);
    const uint32_t b = value;
    const uint32_t word = b | (b << 8) | (b << 16) | (b << 24);
    const uint4 pat = make_uint4(word, word, word, word);
    for (uint64_t j = i; j < nvec; j += stride) v[j] = pat;
    const uint64_t tail0 = h + nvec * 16;
    for (uint64_t j = tail0 + i; j < n; j += stride) dst[j] = value;
}

__global__ void count_mismatch_kernel(const uint8_t* __restrict__ p, uint64_t n, uint8_t value,
                                      unsigned long long* __restrict__ count) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    unsigned long long local = 0;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        local += (p[i] != value);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
    if ((threadIdx.x & 31) == 0 && local) atomicAdd(count, local);
}

unsigned grid_for(uint64_t n, unsigned threads) {
    const uint64_t want = (n + threads * 16ull - 1) / (threads * 16ull);
    const uint64_t cap = (uint64_t)sf::sm_count() * 8;
    uint64_t g = want < cap ? want : cap;
    return (unsigned)(g ? g : 1);
}

}  // namespace

extern "C" const char* sf_version(void) { return "0.1.0+sm_100a"; }

extern "C" int sf_device_info_get(int32_t device, sf_device_info* out, char* err, uint64_t cap) {
    if (!out) return sf::fail(SF_EINVAL, err, cap, "sf_device_info_get: null output");
    cudaDeviceProp p;
    cudaError_t e = cudaGetDeviceProperties(&p, device);
    if (e != cudaSuccess) return sf::fail(SF_EDEVICE, err, cap, "cudaGetDeviceProperties(%d): %s", device, cudaGetErrorString(e));
    out->device = device;
    out->cc_major = p.major;
    out->cc_minor = p.minor;
    out->sm_count = p.multiProcessorCount;
    out->global_mem_bytes = (int64_t)p.totalGlobalMem;
    out->l2_bytes = (int64_t)p.l2CacheSize;
    out->max_smem_per_block_optin = (int32_t)p.sharedMemPerBlockOptin;
    out->max_threads_per_block = p.maxThreadsPerBlock;
    int clk = 0, mclk = 0, bus = 0;
    cudaDeviceGetAttribute(&clk, cudaDevAttrClockRate, device);
    cudaDeviceGetAttribute(&mclk, cudaDevAttrMemoryClockRate, device);
    cudaDeviceGetAttribute(&bus, cudaDevAttrGlobalMemoryBusWidth, device);
    out->clock_khz = clk;
    out->mem_clock_khz = mclk;
    out->mem_bus_width_bits = bus;
    snprintf(out->name, sizeof(out->name), "%s", p.name);
    return SF_OK;
}

extern "C" int sf_fill_bytes(void* dst, uint64_t nbytes, int32_t value, void* stream, char* err, uint64_t cap) {
    if (nbytes == 0) return SF_OK;
    if (!dst || value < 0 || value > 255) return sf::fail(SF_EINVAL, err, cap, "sf_fill_bytes: bad arguments");
    fill_bytes_kernel<<<grid_for(nbytes, 256), 256, 0, (cudaStream_t)stream>>>((uint8_t*)dst, nbytes, (uint8_t)value);
    return sf::check_launch("sf_fill_bytes", err, cap);
}

extern "C" int sf_count_mismatch(const void* ptr, uint64_t nbytes, int32_t value, uint64_t* count_dev, void* stream,
                                 char* err, uint64_t cap) {
    if (nbytes == 0) return SF_OK;
    if (!ptr || !count_dev || value < 0 || value > 255) return sf::fail(SF_EINVAL, err, cap, "sf_count_mismatch: bad arguments");
    count_mismatch_kernel<<<grid_for(nbytes, 256), 256, 0, (cudaStream_t)stream>>>(
        (const uint8_t*)ptr, nbytes, (uint8_t)value, (unsigned long long*)count_dev);
    return sf::check_launch("sf_count_mismatch", err, cap);
}

extern "C" int32_t sf_op_nargs(int32_t op) {
    switch (op) {
        case SF_OP_RMSNORM: return 3;
        case SF_OP_GEMM_NT: return 3;
        case SF_OP_GEMM_NN: return 4;
        case SF_OP_SILU: return 2;
        case SF_OP_SWIGLU: return 3;
        case SF_OP_SOFTMAX: return 2;
        case SF_OP_REDUCTION_SUM: return 2;
        case SF_OP_ROPE: return 2;
        case SF_OP_BITDELTA: return 3;
        case SF_OP_BITDELTA_BASE: return 5;
        case SF_OP_ATTENTION: return 4;
        case SF_OP_KDA: return 13;
        case SF_OP_KDA_GATED: return 10;
        case SF_OP_MAMBA2: return 8;
        case SF_OP_RELU: return 2;
        case SF_OP_SIGMOID: return 2;
        case SF_OP_SIGMOID_SHIFT: return 2;
        case SF_OP_LION: return 5;
        case SF_OP_GEMV: return 3;
        case SF_OP_GEMM_SILU: return 4;
        case SF_OP_KDA_FIXED: return 14;
        default: return 0;
    }
}

static int dispatch(const sf_op_desc* d, const void* const* a, cudaStream_t s, char* err, uint64_t cap) {
    switch (d->op) {
        case SF_OP_RMSNORM:
            return sf_rmsnorm_launch(a[0], a[1], (void*)a[2], d->dims[0], d->dims[1], (float)d->attrs[0], d->dtype,
                                     d->variant, s, err, cap);
        case SF_OP_GEMM_NT:
            return sf_gemm_nt_launch(a[0], a[1], (void*)a[2], d->dims[0], d->dims[1], d->dims[2], d->dtype, d->variant, s, err, cap);
        case SF_OP_GEMM_NN:
            return sf_gemm_nn_launch(a[0], a[1], (void*)a[2], d->dims[0], d->dims[1], d->dims[2], d->dtype, d->variant, (void*)a[3],
                                     (uint64_t)d->dims[3], s, err, cap);
        case SF_OP_SILU:
            return sf_silu_launch(a[0], (void*)a[1], d->dims[0], d->dtype, d->variant, s, err, cap);
        case SF_OP_SWIGLU:
            return sf_swiglu_launch(a[0], a[1], (void*)a[2], d->dims[0], d->dtype, d->variant, s, err, cap);
        case SF_OP_SOFTMAX:
            return sf_softmax_launch(a[0], (void*)a[1], d->dims[0], d->dims[1], d->dtype, d->variant, s, err, cap);
        case SF_OP_REDUCTION_SUM:
            return sf_reduction_sum_launch(a[0], (void*)a[1], d->dims[0], d->dims[1], d->dtype, d->variant, s, err, cap);
        case SF_OP_ROPE:
            return sf_rope_launch(a[0], (void*)a[1], d->dims[0], d->dims[1], d->dims[2], d->dims[3], d->attrs[0], d->dtype,
                                  d->variant, s, err, cap);
        case SF_OP_BITDELTA:
            return sf_bitdelta_launch(a[0], a[1], (void*)a[2], d->dims[0], d->dims[1], d->dims[2], (float)d->attrs[0], d->dtype,
                                      d->variant, s, err, cap);
        case SF_OP_BITDELTA_BASE:
            return sf_bitdelta_base_launch(a[0], a[1], a[2], a[3], (void*)a[4], d->dims[0], d->dims[1], d->dims[2], d->dtype,
                                           d->variant, s, err, cap);
        case SF_OP_ATTENTION:
            return sf_attention_launch(a[0], a[1], a[2], (void*)a[3], d->dims[0], d->dims[1], d->dims[2], d->dims[3], (float)d->attrs[0],
                                       d->flags & 1, d->dtype, d->variant, s, err, cap);
        case SF_OP_KDA:
            return sf_kda_launch(a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7], a[8], a[9], (void*)a[10], (void*)a[11], d->dims[0],
                                 d->dims[1], d->dims[2], (float)d->attrs[0], d->dtype, d->variant, d->dims[3], (void*)a[12],
                                 (uint64_t)d->dims[4], s, err, cap);
        case SF_OP_KDA_GATED:
            return sf_kda_gated_launch(a[0], a[1], a[2], a[3], a[4], a[5], a[6], (void*)a[7], (void*)a[8], d->dims[0], d->dims[1],
                                       d->dims[2], (float)d->attrs[0], d->dtype, d->variant, d->dims[3], (void*)a[9],
                                       (uint64_t)d->dims[4], s, err, cap);
        case SF_OP_MAMBA2:
            return sf_mamba2_launch(a[0], a[1], a[2], a[3], a[4], a[5], a[6], (void*)a[7], d->dims[0], d->dims[1], d->dims[2], d->dims[3],
                                    d->dims[4], d->dims[5], d->dtype, d->variant, s, err, cap);
        case SF_OP_RELU:
            return sf_relu_launch(a[0], (void*)a[1], d->dims[0], d->dtype, d->variant, s, err, cap);
        case SF_OP_SIGMOID:
            return sf_sigmoid_launch(a[0], (void*)a[1], d->dims[0], d->dtype, d->variant, s, err, cap);
        case SF_OP_SIGMOID_SHIFT:
            return sf_sigmoid_shift_launch(a[0], (void*)a[1], d->dims[0], d->dtype, d->variant, s, err, cap);
        case SF_OP_LION:
            return sf_lion_launch(a[0], a[1], a[2], (void*)a[3], (void*)a[4], d->dims[0], d->attrs[0], d->attrs[1], d->attrs[2],
                                  d->attrs[3], d->dtype, d->variant, s, err, cap);
        case SF_OP_GEMV:
            return sf_gemv_launch(a[0], a[1], (void*)a[2], d->dims[0], d->dims[1], d->dtype, d->variant, s, err, cap);
        case SF_OP_GEMM_SILU:
            return sf_gemm_silu_launch(a[0], a[1], (void*)a[2], d->dims[0], d->dims[1], d->dims[2], d->dtype, d->variant, (void*)a[3],
                                       (uint64_t)d->dims[3], s, err, cap);
        case SF_OP_KDA_FIXED:
            return sf_kda_fixed_launch(a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7], a[8], (void*)a[9], (void*)a[10], (void*)a[11],
                                       (void*)a[12], d->dims[0], d->dims[1], d->dims[2], (float)d->attrs[0], d->dtype, d->variant, s,
                                       err, cap);
        default:
            return sf::fail(SF_EINVAL, err, cap, "unknown op %d", d->op);
    }
}

extern "C" int sf_run_op(const sf_op_desc* desc, const void* const* args, uint64_t nargs, void* stream, char* err,
                         uint64_t cap) {
    if (!desc || !args) return sf::fail(SF_EINVAL, err, cap, "sf_run_op: null descriptor or arguments");
    const int32_t want = sf_op_nargs(desc->op);
    if (want == 0) return sf::fail(SF_EINVAL, err, cap, "sf_run_op: unknown op %d", desc->op);
    if ((uint64_t)want != nargs) return sf::fail(SF_EINVAL, err, cap, "sf_run_op: op %d takes %d tensors, got %llu", desc->op, want, (unsigned long long)nargs);
    return dispatch(desc, args, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_run_batch(const sf_op_desc* desc, const void* const* args, uint64_t nargs, uint64_t nsets,
                            uint64_t iters, int32_t use_graph, void* stream_ptr, double* gpu_s, char* err, uint64_t cap) {
    if (!desc || !args || !gpu_s || nsets == 0 || iters == 0) return sf::fail(SF_EINVAL, err, cap, "sf_run_batch: bad arguments");
    const int32_t want = sf_op_nargs(desc->op);
    if (want == 0 || (uint64_t)want != nargs) return sf::fail(SF_EINVAL, err, cap, "sf_run_batch: op %d takes %d tensors, got %llu", desc->op, want, (unsigned long long)nargs);
    cudaStream_t stream = (cudaStream_t)stream_ptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int rc = SF_OK;
    cudaError_t ce;
    if ((ce = cudaEventCreate(&e0)) != cudaSuccess || (ce = cudaEventCreate(&e1)) != cudaSuccess) {
        rc = sf::fail(SF_EDEVICE, err, cap, "cudaEventCreate: %s", cudaGetErrorString(ce));
        goto done;
    }
    if (use_graph) {
        // Capture the launches once (untimed) on a private stream, then time one graph launch.
        cudaStream_t cs;
        if ((ce = cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking)) != cudaSuccess) {
            rc = sf::fail(SF_EDEVICE, err, cap, "cudaStreamCreate: %s", cudaGetErrorString(ce));
            goto done;
        }
        ce = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
        if (ce == cudaSuccess) {
            for (uint64_t i = 0; i < iters && rc == SF_OK; ++i) {
                rc = dispatch(desc, args + (i % nsets) * nargs, cs, err, cap);
            }
            cudaError_t ce2 = cudaStreamEndCapture(cs, &graph);
            if (rc == SF_OK && ce2 != cudaSuccess) rc = sf::fail(SF_EDEVICE, err, cap, "graph capture: %s", cudaGetErrorString(ce2));
        } else {
            rc = sf::fail(SF_EDEVICE, err, cap, "cudaStreamBeginCapture: %s", cudaGetErrorString(ce));
        }
        cudaStreamDestroy(cs);
        if (rc != SF_OK) goto done;
        if ((ce = cudaGraphInstantiate(&exec, graph, 0)) != cudaSuccess) {
            rc = sf::fail(SF_EDEVICE, err, cap, "cudaGraphInstantiate: %s", cudaGetErrorString(ce));
            goto done;
        }
        if ((ce = cudaGraphUpload(exec, stream)) != cudaSuccess) {
            rc = sf::fail(SF_EDEVICE, err, cap, "cudaGraphUpload: %s", cudaGetErrorString(ce));
            goto done;
        }
        cudaEventRecord(e0, stream);
        ce = cudaGraphLaunch(exec, stream);
        cudaEventRecord(e1, stream);
        if (ce != cudaSuccess) {
            rc = sf::fail(SF_EDEVICE, err, cap, "cudaGraphLaunch: %s", cudaGetErrorString(ce));
            goto done;
        }
    } else {
        cudaEventRecord(e0, stream);
        for (uint64_t i = 0; i < iters && rc == SF_OK; ++i) {
            rc = dispatch(desc, args + (i % nsets) * nargs, stream, err, cap);
        }
        cudaEventRecord(e1, stream);
        if (rc != SF_OK) goto done;
    }
    if ((ce = cudaEventSynchronize(e1)) != cudaSuccess) {
        rc = sf::fail(SF_EDEVICE, err, cap, "batch execution: %s", cudaGetErrorString(ce));
        goto done;
    }
    {
        float ms = 0.f;
        if ((ce = cudaEventElapsedTime(&ms, e0, e1)) != cudaSuccess) {
            rc = sf::fail(SF_EDEVICE, err, cap, "cudaEventElapsedTime: %s", cudaGetErrorString(ce));
            goto done;
        }
        *gpu_s = (double)ms * 1e-3;
    }
done:
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    return rc;
}
