// Host helpers for the TMA-fed kernels (tma_host.cu).
#pragma once

#include <cuda.h>
#include <atomic>
#include <stdint.h>

namespace sf {

// 2-D tiled tensor map over a row-major matrix [rows, inner] with `row_stride_bytes` between rows,
// box = box_inner x box_rows elements, 128-byte swizzle, zero fill out of bounds.  Cached.
int tmap_2d(CUtensorMap* out, const void* base, int64_t rows, int64_t inner, int64_t row_stride_bytes, int box_inner, int box_rows,
            int elem_bytes, bool bf16, char* err, uint64_t cap);

// 3-D tiled 16-bit tensor map over [d2, d1, d0] (d0 innermost) with the given byte strides of
// dims 1 and 2, box = box0 x box1 x box2, 128-byte swizzle, zero fill out of bounds.  Cached.
int tmap_3d(CUtensorMap* out, const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t stride1_bytes, int64_t stride2_bytes,
            int box0, int box1, int box2, bool bf16, char* err, uint64_t cap);

// 3-D tiled fp32 tensor map over [d2, d1, d0] (d0 innermost), box = box0 x box1 x box2 with
// box0 = 32 (one 128-byte swizzle row), 128-byte swizzle, zero fill out of bounds.  Cached.
int tmap_3d_f32(CUtensorMap* out, const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t stride1_bytes, int64_t stride2_bytes,
                int box0, int box1, int box2, char* err, uint64_t cap);

// K-major 16-bit operand [rows, K]: box of 64 elements (one 128-byte swizzle row) x box_rows.
int tmap_kmajor(CUtensorMap* out, const void* base, int64_t rows, int64_t K, int box_rows, bool bf16, char* err, uint64_t cap);

// True the first time it is called for the current device with this mask (per-kernel attribute
// set-up such as the dynamic shared-memory limit).
bool once_per_device(std::atomic<uint64_t>& mask);

}  // namespace sf
