// decode_sm100.cu -- decode attention (one query token per (batch, head))
// over a padded bf16 KV cache, split over 256-key chunks (split-KV).
//
// The step is HBM-bound: every valid K and V byte is read exactly once and
// nothing else of size is touched.  Per CTA (one (batch, head, chunk)):
//   1. one thread issues two bulk copies (cp.async.bulk, async proxy) of
//      exactly the chunk's valid K rows and V rows into shared memory -- the
//      padding past kv_lens[b] is never read;
//   2. scores: 8 lanes per key, 16-byte smem loads, 3-step xor-shuffle dot
//      reduction; the query is pre-scaled by scale*log2(e);
//   3. chunk max / sum with warp shuffles, p = exp2(s - m);
//   4. P.V: 8 lanes x 8 columns per key row, 4 rows per warp step, shuffle +
//      smem reduction over key groups and warps;
//   5. the partial (m, l, acc[64]) of the chunk goes to the workspace.
// A second kernel merges the partials of each (batch, head) (one warp each)
// and writes the f32 output.  K/V loads for the score phase overlap the V
// transfer (separate barriers), and ~3 CTAs per SM keep loads in flight.
#include <math.h>

#include <mutex>
#include <vector>

#include "sm100_ptx.cuh"
#include "wfattn_internal.h"

namespace wfattn {
namespace {

constexpr int kChunk = 256;  // keys per CTA
constexpr int kD = 64;
constexpr int kThreads = 128;
constexpr uint32_t kRowBytes = kD * 2;
constexpr int kPartFloats = kD + 2;  // acc[64], m, l

struct DecSmem {
  uint8_t k[kChunk * kRowBytes];
  uint8_t v[kChunk * kRowBytes];
  float s[kChunk];
  float oacc[4][kD];
  float red[8];
  uint64_t bar_k, bar_v;
};

struct DecParams {
  int64_t H, max_len;
  int nch;  // chunks per (batch, head) = ceil(max_len / kChunk)
  const char *q, *k, *v;
  int64_t qs_b, qs_h, ks_b, ks_h, vs_b, vs_h;  // element strides (seq stride is kD)
  const int32_t *kv_lens;
  float *part;  // [B*H*nch][kPartFloats]
  float scale_log2;
  unsigned int *status;
};

__device__ __forceinline__ int64_t clamp_len(int32_t L, int64_t max_len, unsigned int *status) {
  if (L < 1 || L > max_len) {
    if (status) atomicOr(status, kDevBadLengthMask);
    return L < 1 ? 0 : max_len;
  }
  return L;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4 &w, float (&f)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}

__global__ void __launch_bounds__(kThreads) decode_split_kernel(const DecParams p) {
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  DecSmem &sm = *reinterpret_cast<DecSmem *>(dsm_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (ptx::timeout_flagged(p.status)) return;  // sticky until the host clears it
  const int64_t bh = blockIdx.x / p.nch;
  const int c = blockIdx.x % p.nch;
  const int64_t b = bh / p.H, h = bh % p.H;
  const int64_t L = clamp_len(p.kv_lens[b], p.max_len, threadIdx.x == 0 ? p.status : nullptr);
  const int64_t t0 = (int64_t)c * kChunk;
  if (t0 >= L) return;  // no valid keys in this chunk; the combine skips it
  const int n = (int)imin64(kChunk, L - t0);

  const uint32_t bar_k = ptx::smem_u32(&sm.bar_k), bar_v = ptx::smem_u32(&sm.bar_v);
  if (threadIdx.x == 0) {
    ptx::mbar_init(bar_k, 1);
    ptx::mbar_init(bar_v, 1);
    ptx::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t bytes = (uint32_t)n * kRowBytes;
    const char *ksrc = p.k + 2 * (b * p.ks_b + h * p.ks_h + t0 * kD);
    const char *vsrc = p.v + 2 * (b * p.vs_b + h * p.vs_h + t0 * kD);
    ptx::mbar_arrive_expect_tx(bar_k, bytes);
    ptx::bulk_load(ptx::smem_u32(sm.k), ksrc, bytes, bar_k);
    ptx::mbar_arrive_expect_tx(bar_v, bytes);
    ptx::bulk_load(ptx::smem_u32(sm.v), vsrc, bytes, bar_v);
  }

  // Query slice of this lane group: columns [8g, 8g+8), pre-scaled.
  const int g = lane & 7, sub = lane >> 3;
  float qf[8];
  {
    const uint4 w = *reinterpret_cast<const uint4 *>(p.q + 2 * (b * p.qs_b + h * p.qs_h) + g * 16);
    bf16x8_to_f32(w, qf);
#pragma unroll
    for (int i = 0; i < 8; ++i) qf[i] *= p.scale_log2;
  }

  // CTA-uniform outcome: every thread takes the same path through the
  // barriers and full-warp shuffles below.
  bool ok = __syncthreads_and(ptx::mbar_wait(bar_k, 0, p.status)) != 0;
  // ---- scores: keys t = 4*warp + sub + 16*i.  The loop bound depends on the
  // warp only, so all 32 lanes run the same iterations and reach every
  // full-mask shuffle together; lanes past the end of the chunk just idle.
  for (int base = warp * 4; ok && base < n; base += 16) {
    const int t = base + sub;
    float d = 0.f;
    if (t < n) {
      const uint4 w = *reinterpret_cast<const uint4 *>(sm.k + t * kRowBytes + g * 16);
      float kf[8];
      bf16x8_to_f32(w, kf);
#pragma unroll
      for (int i = 0; i < 8; ++i) d = fmaf(qf[i], kf[i], d);
    }
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    d += __shfl_xor_sync(0xffffffffu, d, 4);
    if (g == 0 && t < n) sm.s[t] = d;
  }
  __syncthreads();

  // ---- chunk max and exp2
  float mx = -INFINITY;
  for (int t = threadIdx.x; t < n; t += kThreads) mx = fmaxf(mx, sm.s[t]);
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, sh));
  if (lane == 0) sm.red[warp] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(sm.red[0], sm.red[1]), fmaxf(sm.red[2], sm.red[3]));
  float sum = 0.f;
  for (int t = threadIdx.x; t < n; t += kThreads) {
    const float e = ptx::ex2_approx(sm.s[t] - mx);
    sm.s[t] = e;
    sum += e;
  }
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, sh);
  if (lane == 0) sm.red[4 + warp] = sum;
  __syncthreads();

  // ---- P.V
  ok = __syncthreads_and(ok && ptx::mbar_wait(bar_v, 0, p.status)) != 0;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int t = warp * 4 + sub; ok && t < n; t += 16) {
    const float pt = sm.s[t];
    const uint4 w = *reinterpret_cast<const uint4 *>(sm.v + t * kRowBytes + g * 16);
    float vf[8];
    bf16x8_to_f32(w, vf);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = fmaf(pt, vf[i], acc[i]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 8);
    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 16);
  }
  if (sub == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) sm.oacc[warp][g * 8 + i] = acc[i];
  }
  __syncthreads();
  float *part = p.part + ((size_t)bh * p.nch + c) * kPartFloats;
  if (threadIdx.x < kD) {
    const int d = threadIdx.x;
    part[d] = sm.oacc[0][d] + sm.oacc[1][d] + sm.oacc[2][d] + sm.oacc[3][d];
  } else if (threadIdx.x == kD) {
    part[kD] = ok ? mx : -INFINITY;
    part[kD + 1] = ok ? (sm.red[4] + sm.red[5] + sm.red[6] + sm.red[7]) : 0.f;
  }
  if (!ok && threadIdx.x == 0) {
    // Drain: both bulk copies must land before the CTA releases its shared memory.
    ptx::mbar_wait_drain(bar_k, 0);
    ptx::mbar_wait_drain(bar_v, 0);
  }
}

struct CombineParams {
  int64_t BH, H, max_len;
  int nch;
  const int32_t *kv_lens;
  const float *part;
  float *o;
  int64_t os_b, os_h;
};

// One warp per (batch, head): merge the chunk partials, write f32 output.
__global__ void __launch_bounds__(128) decode_combine_kernel(const CombineParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t bh = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (bh >= p.BH) return;
  const int64_t b = bh / p.H, h = bh % p.H;
  int64_t L = p.kv_lens[b];
  L = L < 1 ? 0 : (L > p.max_len ? p.max_len : L);
  const int nc = (int)((L + kChunk - 1) / kChunk);
  const float *part = p.part + (size_t)bh * p.nch * kPartFloats;
  float M = -INFINITY;
  for (int c = lane; c < nc; c += 32) M = fmaxf(M, part[(size_t)c * kPartFloats + kD]);
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
  float o0 = 0.f, o1 = 0.f, l = 0.f;
  for (int c = 0; c < nc; ++c) {
    const float *pc = part + (size_t)c * kPartFloats;
    const float mc = pc[kD];
    const float w = mc == -INFINITY ? 0.f : ptx::ex2_approx(mc - M);
    const float2 a = *reinterpret_cast<const float2 *>(pc + 2 * lane);
    o0 = fmaf(a.x, w, o0);
    o1 = fmaf(a.y, w, o1);
    l = fmaf(pc[kD + 1], w, l);
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  float *dst = p.o + b * p.os_b + h * p.os_h;
  *reinterpret_cast<float2 *>(dst + 2 * lane) = make_float2(o0 * inv, o1 * inv);
}

std::mutex g_scratch_mutex;
std::vector<void *> g_scratch_addr;  // per device ordinal; nullptr until set up

}  // namespace

// Scratch of the allocation-free decode entry point: a file-scope device
// array, so the library never has to call cudaMalloc for it.  Every device
// that loads this module holds it until the process exits.
static __device__ __align__(256) unsigned char g_decode_scratch[kDecodeNoAllocScratchBytes];

// Device address of g_decode_scratch on the current device.  Host code cannot
// pass the symbol itself to a kernel (on the host it names a host-side
// stand-in), so the address is looked up once per device, with that device
// current, and cached.
cudaError_t decode_noalloc_scratch(void **ptr) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if ((int)g_scratch_addr.size() <= dev) g_scratch_addr.resize(dev + 1, nullptr);
  if (!g_scratch_addr[dev]) {
    void *addr = nullptr;
    err = cudaGetSymbolAddress(&addr, g_decode_scratch);
    if (err != cudaSuccess) return err;
    g_scratch_addr[dev] = addr;
  }
  *ptr = g_scratch_addr[dev];
  return cudaSuccess;
}

size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t max_len, int64_t) {
  const int64_t nch = (max_len + kChunk - 1) / kChunk;
  return (size_t)(B * H * nch) * kPartFloats * sizeof(float);
}

cudaError_t launch_decode_bf16(const DecodeArgs &a, const DeviceInfo &dev, cudaStream_t stream) {
  if (a.ks.s != kD || a.vs.s != kD) return cudaErrorInvalidValue;  // rows must be contiguous
  DecParams p;
  p.H = a.H;
  p.max_len = a.max_len;
  p.nch = (int)((a.max_len + kChunk - 1) / kChunk);
  p.q = static_cast<const char *>(a.q);
  p.k = static_cast<const char *>(a.k);
  p.v = static_cast<const char *>(a.v);
  p.qs_b = a.qs.b;
  p.qs_h = a.qs.h;
  p.ks_b = a.ks.b;
  p.ks_h = a.ks.h;
  p.vs_b = a.vs.b;
  p.vs_h = a.vs.h;
  p.kv_lens = a.kv_lens;
  p.part = static_cast<float *>(a.workspace);
  p.scale_log2 = (float)((double)a.scale * 1.4426950408889634);
  p.status = dev.status;
  const int64_t blocks = a.B * a.H * p.nch;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  const size_t smem = sizeof(DecSmem);
  cudaError_t err = cudaFuncSetAttribute(decode_split_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err != cudaSuccess) return err;
  decode_split_kernel<<<(unsigned)blocks, kThreads, smem, stream>>>(p);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  CombineParams cp;
  cp.BH = a.B * a.H;
  cp.H = a.H;
  cp.max_len = a.max_len;
  cp.nch = p.nch;
  cp.kv_lens = a.kv_lens;
  cp.part = p.part;
  cp.o = a.o;
  cp.os_b = a.os.b;
  cp.os_h = a.os.h;
  decode_combine_kernel<<<(unsigned)((cp.BH + 3) / 4), 128, 0, stream>>>(cp);
  return cudaGetLastError();
}

}  // namespace wfattn
