// Internal launch interface between the C ABI layer (wfattn_api.cu) and the
// kernel translation units.  Every launcher returns a cudaError_t from the
// launch; argument validation has already happened in the API layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace wfattn {

// Device-side status bits written by kernels whose bounded waits expired.
enum DeviceStatusBits : unsigned int {
  kDevTimeoutMask = 1u,
  kDevBadLengthMask = 2u,  // a device-side length (decode kv_lens) was out of range
};

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t imax64(int64_t a, int64_t b) { return a > b ? a : b; }

// Strided [B, H, S, D] view (element strides, unit head_dim stride).
struct Strides3 {
  int64_t b, h, s;
};

constexpr int kMaxOutputPeers = 8;

struct PrefillArgs {
  int64_t B, H, Sq, Sk, D;
  const void *q, *k, *v;
  void *o;
  Strides3 qs, ks, vs, os;
  float scale;  // already resolved (> 0)
  int causal;
  // bf16 two-tile kernel only: when n_peers > 0 the output goes to every one of
  // these buffers (same shape and strides os, possibly on other GPUs) instead of o.
  void *const *o_peers = nullptr;
  int n_peers = 0;
  // bf16 two-tile kernel only: when set, a multicast (NVLS) address of the
  // output (shape and strides os) bound on every GPU of the gather; each output
  // row is written once through it and lands in every GPU's buffer.
  void *o_mc = nullptr;
};

struct DecodeArgs {
  bool f32 = false;  // q, k, v are f32 (else bf16)
  int64_t B, H, D, max_len;
  const void *q;  // [B, H, D]
  Strides3 qs;    // s unused
  const void *k, *v;
  Strides3 ks, vs;
  const int32_t *kv_lens;
  float *o;     // f32 [B, H, D]
  Strides3 os;  // s unused
  float scale;
  void *workspace;
  size_t workspace_bytes;
};

struct DeviceInfo {
  int device;
  int sm_count;
  int cc_major, cc_minor;
  size_t smem_optin;
  unsigned int *status;  // device address of the status word
};

// Sets cudaFuncAttributeMaxDynamicSharedMemorySize of `func` on the current
// device to `bytes` the first time it is asked for that (func, device, bytes)
// and remembers it, so launches do not repeat the driver call.
cudaError_t ensure_smem_attr(const void *func, int bytes, int device);

cudaError_t launch_prefill_f32(const PrefillArgs &a, const DeviceInfo &dev, cudaStream_t stream);
// f32 prefill on the tensor cores (3xTF32 split, head_dim 64): whether the
// views suit its TMA loads and vector stores, and its launcher.
bool prefill_f32_tc_supported(const PrefillArgs &a);
cudaError_t launch_prefill_f32_tc(const PrefillArgs &a, const DeviceInfo &dev,
                                  cudaStream_t stream);
// bf16 prefill: one 128-row query tile per CTA (2 CTAs per SM) ...
cudaError_t launch_prefill_bf16_1q(const PrefillArgs &a, const DeviceInfo &dev,
                                   cudaStream_t stream);
// ... or two 128-row tiles per CTA sharing K/V (1 CTA per SM).
cudaError_t launch_prefill_bf16_2q(const PrefillArgs &a, const DeviceInfo &dev,
                                   cudaStream_t stream);

// Decode shapes the kernels index safely: sizes >= 1, max_len <= 2^31 - 1,
// B*H <= 2^31 - 1 (checked without overflow).
bool decode_shape_ok(int64_t B, int64_t H, int64_t max_len);
// Workspace bytes of a decode call over a bf16 (f32 = false) or f32 cache
// (0 when decode_shape_ok fails).
size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t max_len, int64_t D, bool f32);
cudaError_t launch_decode(const DecodeArgs &a, const DeviceInfo &dev, cudaStream_t stream);

// Size of the static device scratch behind wfattn_decode_noalloc (8 MiB).
constexpr size_t kDecodeNoAllocScratchBytes = size_t(8) << 20;
// Device address of that scratch on the current device (looked up on first use).
cudaError_t decode_noalloc_scratch(void **ptr);

}  // namespace wfattn
