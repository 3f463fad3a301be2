// Tensor maps (TMA descriptors) for the caches, encoded on the host through
// the driver entry point the runtime hands out, so the library does not link
// libcuda directly.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rl {

// A 2-D bf16 tensor of `rows` rows of `cols` elements (row pitch
// `row_bytes`, a multiple of 16), read in boxes of box_rows x box_cols with
// the 128-byte swizzle (box_cols * 2 <= 128).  Returns cudaErrorInvalidValue
// when the driver refuses the encoding.
cudaError_t encode_bf16_2d(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                           uint64_t row_bytes, uint32_t box_rows, uint32_t box_cols);

// A 3-D bf16 tensor [d2][d1][d0] (d0 contiguous, strides in bytes for d1 and
// d2, multiples of 16), read in boxes of b2 x b1 x b0 with the 128-byte
// swizzle (b0 * 2 <= 128).
cudaError_t encode_bf16_3d(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1,
                           uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                           uint32_t b0, uint32_t b1, uint32_t b2);

// A 2-D f32 tensor of `rows` rows of `cols` elements (row pitch
// `row_bytes`, a multiple of 16), moved in boxes of box_rows x box_cols with
// the 128-byte swizzle (box_cols * 4 <= 128), loaded and stored.
cudaError_t encode_f32_2d(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                          uint64_t row_bytes, uint32_t box_rows, uint32_t box_cols);

}  // namespace rl
