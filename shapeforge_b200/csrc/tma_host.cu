// Host-side TMA descriptor encoding shared by the tensor-core kernels, with a cache.
//
// cuTensorMapEncodeTiled is resolved once through cudaGetDriverEntryPoint (the library does not
// link libcuda).  Encoding a descriptor costs host time on every launch; timed batches of short
// kernels would become host-bound, so descriptors are cached by their full parameter set.
#include "sf_common.cuh"
#include "tma_host.cuh"

#include <cudaTypedefs.h>
#include <mutex>
#include <unordered_map>

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

struct Key {
    uintptr_t base;
    int64_t rows, inner, stride;
    int box_inner, box_rows, dtype, swizzle;
    bool operator==(const Key& o) const {
        return base == o.base && rows == o.rows && inner == o.inner && stride == o.stride && box_inner == o.box_inner &&
               box_rows == o.box_rows && dtype == o.dtype && swizzle == o.swizzle;
    }
};

struct KeyHash {
    size_t operator()(const Key& k) const {
        uint64_t h = k.base * 0x9E3779B97F4A7C15ull;
        for (int64_t v : {k.rows, k.inner, k.stride, (int64_t)k.box_inner, (int64_t)k.box_rows, (int64_t)k.dtype, (int64_t)k.swizzle})
            h = (h ^ (uint64_t)v) * 0x100000001B3ull;
        return (size_t)h;
    }
};

std::mutex g_mu;
std::unordered_map<Key, CUtensorMap, KeyHash> g_cache;

}  // namespace

namespace sf {

int tmap_2d(CUtensorMap* out, const void* base, int64_t rows, int64_t inner, int64_t row_stride_bytes, int box_inner, int box_rows,
            int elem_bytes, bool bf16, char* err, uint64_t cap) {
    const int dtype = elem_bytes == 2 ? (bf16 ? 1 : 0) : (elem_bytes == 4 ? 2 : 3);
    const Key key{reinterpret_cast<uintptr_t>(base), rows, inner, row_stride_bytes, box_inner, box_rows, dtype, 128};
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto it = g_cache.find(key);
        if (it != g_cache.end()) {
            *out = it->second;
            return SF_OK;
        }
    }
    auto fn = encode_fn();
    if (!fn) return fail(SF_EDEVICE, err, cap, "cuTensorMapEncodeTiled is unavailable from the driver");
    CUtensorMapDataType t = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    if (dtype == 1) t = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if (dtype == 2) t = CU_TENSOR_MAP_DATA_TYPE_UINT32;
    if (dtype == 3) t = CU_TENSOR_MAP_DATA_TYPE_UINT8;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_stride_bytes};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUtensorMap map;
    CUresult r = fn(&map, t, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SF_EINVAL, err, cap, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (g_cache.size() > 4096) g_cache.clear();
        g_cache.emplace(key, map);
    }
    *out = map;
    return SF_OK;
}

int tmap_3d(CUtensorMap* out, const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t stride1_bytes, int64_t stride2_bytes,
            int box0, int box1, int box2, bool bf16, char* err, uint64_t cap) {
    // Cached under a key that cannot collide with the 2-D entries (swizzle field = -3).
    const Key key{reinterpret_cast<uintptr_t>(base), d1 * 1000003 + d2, d0, stride1_bytes ^ (stride2_bytes << 20), box0,
                  box1 * 4096 + box2, bf16 ? 1 : 0, -3};
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto it = g_cache.find(key);
        if (it != g_cache.end()) {
            *out = it->second;
            return SF_OK;
        }
    }
    auto fn = encode_fn();
    if (!fn) return fail(SF_EDEVICE, err, cap, "cuTensorMapEncodeTiled is unavailable from the driver");
    cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
    cuuint64_t strides[2] = {(cuuint64_t)stride1_bytes, (cuuint64_t)stride2_bytes};
    cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, (cuuint32_t)box2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMap map;
    CUresult r = fn(&map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SF_EINVAL, err, cap, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (g_cache.size() > 4096) g_cache.clear();
        g_cache.emplace(key, map);
    }
    *out = map;
    return SF_OK;
}

int tmap_3d_f32(CUtensorMap* out, const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t stride1_bytes, int64_t stride2_bytes,
                int box0, int box1, int box2, char* err, uint64_t cap) {
    // Cached under a key of its own (dtype field = 2, swizzle field = -4).
    const Key key{reinterpret_cast<uintptr_t>(base), d1 * 1000003 + d2, d0, stride1_bytes ^ (stride2_bytes << 20), box0,
                  box1 * 4096 + box2, 2, -4};
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto it = g_cache.find(key);
        if (it != g_cache.end()) {
            *out = it->second;
            return SF_OK;
        }
    }
    auto fn = encode_fn();
    if (!fn) return fail(SF_EDEVICE, err, cap, "cuTensorMapEncodeTiled is unavailable from the driver");
    cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
    cuuint64_t strides[2] = {(cuuint64_t)stride1_bytes, (cuuint64_t)stride2_bytes};
    cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, (cuuint32_t)box2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUtensorMap map;
    CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SF_EINVAL, err, cap, "cuTensorMapEncodeTiled (3-D fp32) failed (%d)", (int)r);
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (g_cache.size() > 4096) g_cache.clear();
        g_cache.emplace(key, map);
    }
    *out = map;
    return SF_OK;
}

int tmap_kmajor(CUtensorMap* out, const void* base, int64_t rows, int64_t K, int box_rows, bool bf16, char* err, uint64_t cap) {
    return tmap_2d(out, base, rows, K, K * 2, 64, box_rows, 2, bf16, err, cap);
}

bool once_per_device(std::atomic<uint64_t>& mask) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return true;
    const uint64_t bit = 1ull << dev;
    return (mask.fetch_or(bit) & bit) == 0;
}

}  // namespace sf
