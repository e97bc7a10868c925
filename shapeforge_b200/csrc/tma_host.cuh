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

// K-major 16-bit operand [rows, K]: box of 64 elements (one 128-byte swizzle row) x box_rows.
int tmap_kmajor(CUtensorMap* out, const void* base, int64_t rows, int64_t K, int box_rows, bool bf16, char* err, uint64_t cap);

// True the first time it is called for the current device with this mask (per-kernel attribute
// set-up such as the dynamic shared-memory limit).
bool once_per_device(std::atomic<uint64_t>& mask);

}  // namespace sf
