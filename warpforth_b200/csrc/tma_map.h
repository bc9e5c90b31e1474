// TMA tensor-map construction shared by the bf16 prefill kernels.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "wfattn_internal.h"

namespace wfattn {

// [B, H, S, 64] bf16 view with element strides {b, h, s} (unit head_dim
// stride) -> 4-D tensor map {64, S, H, B}, box {64, 128, 1, 1}, 128-byte
// swizzle, zero fill outside the tensor.  Returns false if the driver entry
// point is unavailable or the encoding is rejected.
bool make_bf16_map_64x128(CUtensorMap *m, const void *base, int64_t B, int64_t H, int64_t S,
                          const Strides3 &st);
// The same with a box of {64, box_rows, 1, 1} (box_rows <= 256).
bool make_bf16_map_64xR(CUtensorMap *m, const void *base, int64_t B, int64_t H, int64_t S,
                        const Strides3 &st, int box_rows);
// Box {box_cols, box_rows, 1, 1} (box_cols * 2 bytes a multiple of 16) with
// 128-byte swizzle (box_cols == 64) or none (shared-memory tile row-major).
bool make_bf16_map(CUtensorMap *m, const void *base, int64_t B, int64_t H, int64_t S,
                   const Strides3 &st, int box_cols, int box_rows, bool swizzle128);

// [B, H, S, 64] f32 view -> 4-D tensor map {64, S, H, B} with a box of
// {32, box_rows, 1, 1} (one 128-byte row of 32 floats) and 128-byte swizzle;
// a 64-column tile is loaded as two boxes (columns 0-31 and 32-63).
bool make_f32_map(CUtensorMap *m, const void *base, int64_t B, int64_t H, int64_t S,
                  const Strides3 &st, int box_rows);

}  // namespace wfattn
