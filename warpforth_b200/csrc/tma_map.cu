// tma_map.cu -- builds TMA tensor maps through the driver entry point that the
// CUDA runtime exposes (no link-time dependency on libcuda).
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "tma_map.h"

namespace wfattn {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void *sym = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &sym, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(sym);
  });
  return fn;
}

}  // namespace

bool make_bf16_map(CUtensorMap *m, const void *base, int64_t B, int64_t H, int64_t S,
                   const Strides3 &st, int box_cols, int box_rows, bool swizzle128) {
  auto enc = encode_fn();
  if (!enc) return false;
  if (box_cols < 8 || box_cols > 64 || box_cols % 8 || (swizzle128 && box_cols != 64))
    return false;
  const cuuint64_t dims[4] = {64, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)st.s * 2, (cuuint64_t)st.h * 2, (cuuint64_t)st.b * 2};
  const cuuint64_t extent[3] = {(cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  // A dimension of extent 1 is never stepped over; give it a legal stride
  // (TMA wants non-zero multiples of 16 bytes).
  for (int i = 0; i < 3; ++i)
    if (extent[i] == 1 && strides[i] == 0) strides[i] = 128;
  const cuuint32_t box[4] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r =
      enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box,
          estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_f32_map(CUtensorMap *m, const void *base, int64_t B, int64_t H, int64_t S,
                  const Strides3 &st, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[4] = {64, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)st.s * 4, (cuuint64_t)st.h * 4, (cuuint64_t)st.b * 4};
  const cuuint64_t extent[3] = {(cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  for (int i = 0; i < 3; ++i)
    if (extent[i] == 1 && strides[i] == 0) strides[i] = 256;
  const cuuint32_t box[4] = {32, (cuuint32_t)box_rows, 1, 1};  // 32 f32 = one 128-byte row
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void *>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_bf16_map_64xR(CUtensorMap *m, const void *base, int64_t B, int64_t H, int64_t S,
                        const Strides3 &st, int box_rows) {
  return make_bf16_map(m, base, B, H, S, st, 64, box_rows, true);
}

bool make_bf16_map_64x128(CUtensorMap *m, const void *base, int64_t B, int64_t H, int64_t S,
                          const Strides3 &st) {
  return make_bf16_map_64xR(m, base, B, H, S, st, 128);
}

}  // namespace wfattn
