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

}  // namespace wfattn
