// Host-side TMA tensor maps shared by the tcgen05 kernels.
#pragma once
#include <cuda.h>
#include <cstdint>

namespace dsv {

// Tensor map of a row-major bf16 matrix [rows, cols] with leading dimension
// `ld` elements; box = 64 columns (128 bytes, 128-byte swizzle) x box_rows.
// Cached by (pointer, shape, box). Defined in gemm_tc.cu.
CUtensorMap make_tmap_bf16(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows);

}  // namespace dsv
