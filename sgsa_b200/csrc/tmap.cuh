// TMA tensor maps over [B, T, H, W] bf16 row tensors.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace sgsa {
// Map viewing a contiguous [B, T, H, W] bf16 tensor as (W, H, B*T) with a box
// of 64 features x 1 head x box_rows tokens and the 128-byte swizzle (one
// 128-byte row per token).  Returns false if the driver refuses the encoding.
bool make_tmap_rows_bf16(CUtensorMap *map, const void *base, int B, int T, int H, int W,
                         int box_rows);
// Map over a row-major fp32 matrix [rows, inner] with a box of 32 columns
// (128 bytes, 128-byte swizzle) x box_rows rows.
bool make_tmap_2d_f32(CUtensorMap *map, const void *base, int inner, long long rows,
                      int box_rows);
}  // namespace sgsa
