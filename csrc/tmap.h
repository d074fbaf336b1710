// Cached 2D TMA descriptor for a row-major bf16 matrix [rows, cols] (leading
// dimension ld elements): box = [64 columns (128 bytes), box_rows], 128-byte
// swizzle, zero fill out of bounds.  Defined in gemm_tcgen05.cu.
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace braid {
CUtensorMap make_tmap(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows);
}
