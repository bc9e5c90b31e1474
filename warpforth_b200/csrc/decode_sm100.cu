// decode_sm100.cu -- decode attention (one query token per (batch, head))
// over a padded KV cache, split over key chunks (split-KV): bf16 caches in
// 256-key chunks, f32 caches (the reference-accurate path, e.g. GPT-2 in f32
// with a KV cache) in 128-key chunks -- 32 KB of K and 32 KB of V per chunk
// either way.
//
// The step is HBM-bound: every valid K and V byte is read exactly once and
// nothing else of size is touched.  A persistent grid (one CTA per SM) walks
// the (chunk, batch, head) work items that hold keys round-robin: chunk-major,
// with the batches ordered by length, so the CTAs' loads differ by at most one
// item (chunks past kv_lens[b] are never visited).  Warp roles, all decoupled
// through mbarriers (no CTA-wide barrier once the loop runs):
//   * producer (warp 16): keeps kStages chunks in flight; for each item it
//     issues bulk copies (cp.async.bulk) of the query row and of exactly the
//     chunk's valid K rows and V rows into a free stage -- the cache padding
//     is never read;
//   * consumers (warps 0-15): warp w takes keys [16w, 16w+16) of the chunk and
//     runs the whole softmax on them in registers: 8 lanes per key (16-byte
//     smem loads, xor-shuffle dot reduction, query pre-scaled by
//     scale*log2(e)), warp max / sum by shuffles, p = exp2(s - m_warp), then
//     P.V with the same lanes (8 columns each); it frees the stage and hands
//     its (m, l, acc[64]) to the merge warp;
//   * merge (warp 17): folds the 16 warp partials of a chunk into the chunk's
//     partial in the workspace.
// A second kernel merges the partials of each (batch, head) (one warp each)
// and writes the f32 output.
#include <math.h>

#include <mutex>
#include <vector>

#include "sm100_ptx.cuh"
#include "wfattn_internal.h"

namespace wfattn {
namespace {

constexpr int kD = 64;
constexpr int kStages = 3;
constexpr int kConsumerWarps = 16;
constexpr int kProducerWarp = kConsumerWarps, kMergeWarp = kConsumerWarps + 1;
constexpr int kThreads = 32 * (kConsumerWarps + 2);
constexpr uint32_t kStageBytes = 32 * 1024;  // K (and V) rows of one chunk
constexpr int kPartFloats = kD + 2;  // acc[64], m, l
constexpr int kMergeStride = kD + 4;  // a warp's row in smem: acc[64], m, l, pad to 16 B
constexpr int kPlanMaxB = 1024;  // batches the in-smem work plan can order

// Per element type of q and the cache: row size, chunk length, and the load of
// the 8 consecutive elements a lane works on, widened to f32.
template <typename T>
struct Elem;
template <>
struct Elem<uint16_t> {  // bf16
  static constexpr uint32_t kRowBytes = kD * 2;
  __device__ static __forceinline__ void load8(const uint8_t *p, float (&f)[8]) {
    const uint4 w = *reinterpret_cast<const uint4 *>(p);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(u[i] << 16);
      f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
    }
  }
};
template <>
struct Elem<float> {
  static constexpr uint32_t kRowBytes = kD * 4;
  __device__ static __forceinline__ void load8(const uint8_t *p, float (&f)[8]) {
    const float4 a = *reinterpret_cast<const float4 *>(p);
    const float4 b = *reinterpret_cast<const float4 *>(p + 16);
    f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w;
    f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
  }
};
// keys per work item: 256 (bf16), 128 (f32)
template <typename T>
struct Chunk {
  static constexpr int value = (int)(kStageBytes / Elem<T>::kRowBytes);
};

struct ItemInfo {
  int64_t bh;
  int c, n;  // chunk index, valid keys (-1: no more work)
};

template <typename T>
struct DecSmem {
  uint8_t k[kStages][kStageBytes];
  uint8_t v[kStages][kStageBytes];
  uint8_t q[kStages][Elem<T>::kRowBytes];
  float merge[kStages][kConsumerWarps][kMergeStride];  // warp partials of a use of a stage
  ItemInfo item[kStages];        // written by the producer, read by the consumers
  ItemInfo merge_item[kStages];  // copy for the merge warp (item[] is refilled earlier)
  uint64_t full[kStages], empty[kStages];       // producer <-> consumers
  uint64_t merged[kStages], merge_free[kStages];  // consumers <-> merge warp
  // Work plan (batch <= kPlanMaxB): batches ordered by chunk count, descending.
  int plan_nch[kPlanMaxB];  // chunks of batch b
  int plan_b[kPlanMaxB];    // batch at each rank
  int plan_len[kPlanMaxB];  // its (clamped) kv length
  uint32_t abort;
};

struct DecParams {
  int64_t B, H, max_len;
  int nch;  // chunks per (batch, head) = ceil(max_len / chunk)
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

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) decode_split_kernel(const DecParams p) {
  constexpr int kChunk = Chunk<T>::value;
  constexpr uint32_t kRowBytes = Elem<T>::kRowBytes;
  constexpr int kKeysPerWarp = kChunk / kConsumerWarps;
  constexpr int kSteps = kKeysPerWarp / 4;  // 4 keys per warp step (8 lanes each)
  extern __shared__ __align__(128) uint8_t dsm_raw[];
  DecSmem<T> &sm = *reinterpret_cast<DecSmem<T> *>(dsm_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (ptx::timeout_flagged(p.status)) return;  // sticky until the host clears it
  volatile uint32_t &abort_flag = sm.abort;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      ptx::mbar_init(ptx::smem_u32(&sm.full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.empty[i]), kConsumerWarps);
      ptx::mbar_init(ptx::smem_u32(&sm.merged[i]), kConsumerWarps);
      ptx::mbar_init(ptx::smem_u32(&sm.merge_free[i]), 1);
    }
    abort_flag = 0;
    ptx::fence_barrier_init();
  }
  // Work plan.  The items with data are (chunk c, batch b, head h) with
  // c < nch_b; enumerated chunk-major with the batches in descending nch_b
  // order, those of chunk c form one contiguous run, so CTA i can take every
  // gridDim-th item with data and the CTAs' loads differ by at most one item.
  const bool planned = p.B <= kPlanMaxB;
  if (planned) {
    for (int b = threadIdx.x; b < p.B; b += kThreads) {
      const int64_t L = clamp_len(p.kv_lens[b], p.max_len, p.status);
      sm.plan_nch[b] = (int)((L + kChunk - 1) / kChunk);
      sm.plan_len[b] = (int)L;
    }
    __syncthreads();
    int rank_of[(kPlanMaxB + kThreads - 1) / kThreads];
#pragma unroll
    for (int i = 0; i < (kPlanMaxB + kThreads - 1) / kThreads; ++i) {
      const int b = threadIdx.x + i * kThreads;
      rank_of[i] = 0;
      if (b < p.B) {
        const int nb = sm.plan_nch[b];
        for (int o = 0; o < p.B; ++o) {
          const int no = sm.plan_nch[o];
          rank_of[i] += (no > nb) || (no == nb && o < b);
        }
      }
    }
    int len_of[(kPlanMaxB + kThreads - 1) / kThreads];
#pragma unroll
    for (int i = 0; i < (kPlanMaxB + kThreads - 1) / kThreads; ++i) {
      const int b = threadIdx.x + i * kThreads;
      len_of[i] = b < p.B ? sm.plan_len[b] : 0;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < (kPlanMaxB + kThreads - 1) / kThreads; ++i) {
      const int b = threadIdx.x + i * kThreads;
      if (b < p.B) {
        sm.plan_b[rank_of[i]] = b;
        sm.plan_len[rank_of[i]] = len_of[i];
      }
    }
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const int64_t BH = p.B * p.H;
      // Planned: items with data only.  Otherwise: every (c, b, h), skipping
      // the chunks past kv_lens[b].
      int64_t total = BH * p.nch;
      if (planned) {
        total = 0;
        for (int r = 0; r < p.B; ++r) total += (int64_t)p.H * sm.plan_nch[sm.plan_b[r]];
      }
      int c_run = 0, r_end = 0;  // planned walk: current chunk, batches with nch > c_run
      int64_t run0 = 0;          // first item of chunk c_run
      if (planned)
        while (r_end < p.B && sm.plan_nch[sm.plan_b[r_end]] > 0) ++r_end;
      int uses = 0;  // stage uses so far (items with data)
      bool ok = true;
      for (int64_t it = blockIdx.x; ok && it < total; it += gridDim.x) {
        int c;
        int64_t b, h, L;
        if (planned) {
          while (it >= run0 + (int64_t)p.H * r_end) {  // next chunk index
            run0 += (int64_t)p.H * r_end;
            ++c_run;
            while (r_end > 0 && sm.plan_nch[sm.plan_b[r_end - 1]] <= c_run) --r_end;
          }
          const int64_t j = it - run0;
          const int r = (int)(j / p.H);
          c = c_run;
          b = sm.plan_b[r];
          h = j % p.H;
          L = sm.plan_len[r];
        } else {
          c = (int)(it / BH);
          b = (it % BH) / p.H;
          h = it % p.H;
          L = clamp_len(p.kv_lens[b], p.max_len, p.status);
          if ((int64_t)c * kChunk >= L) continue;  // no valid keys; the combine skips it
        }
        const int64_t bh = b * p.H + h;
        const int64_t t0 = (int64_t)c * kChunk;
        const int n = (int)imin64(kChunk, L - t0);
        const int st = uses % kStages;
        if (uses >= kStages &&
            !ptx::mbar_wait(ptx::smem_u32(&sm.empty[st]), (uint32_t)(uses / kStages - 1) & 1,
                            p.status)) {
          ok = false;
          break;
        }
        if (abort_flag) {
          ok = false;
          break;
        }
        sm.item[st].bh = bh;
        sm.item[st].c = c;
        sm.item[st].n = n;
        const uint32_t bytes = (uint32_t)n * kRowBytes;
        constexpr int64_t es = sizeof(T);
        const char *qsrc = p.q + es * (b * p.qs_b + h * p.qs_h);
        const char *ksrc = p.k + es * (b * p.ks_b + h * p.ks_h + t0 * kD);
        const char *vsrc = p.v + es * (b * p.vs_b + h * p.vs_h + t0 * kD);
        const uint32_t fb = ptx::smem_u32(&sm.full[st]);
        ptx::mbar_arrive_expect_tx(fb, 2 * bytes + kRowBytes);
        ptx::bulk_load(ptx::smem_u32(sm.q[st]), qsrc, kRowBytes, fb);
        ptx::bulk_load(ptx::smem_u32(sm.k[st]), ksrc, bytes, fb);
        ptx::bulk_load(ptx::smem_u32(sm.v[st]), vsrc, bytes, fb);
        ++uses;
      }
      if (ok) {
        // End marker: a stage whose item has n = -1, published without data.
        const int st = uses % kStages;
        ok = uses < kStages ||
             ptx::mbar_wait(ptx::smem_u32(&sm.empty[st]), (uint32_t)(uses / kStages - 1) & 1,
                            p.status);
        if (ok) {
          sm.item[st].n = -1;
          ptx::mbar_arrive(ptx::smem_u32(&sm.full[st]));
        }
      }
      if (!ok) {
        abort_flag = 1;
        // Drain: every copy this thread issued must land before the CTA exits.
        for (int i = uses < kStages ? uses : kStages; i > 0; --i) {
          const int u = uses - i;
          ptx::mbar_wait_drain(ptx::smem_u32(&sm.full[u % kStages]), (uint32_t)(u / kStages) & 1);
        }
      }
    }
    return;
  }

  if (warp == kMergeWarp) {
    // ------------------------------------------------------------ merge warp
    // Lane l folds columns 2l, 2l+1; lane 0 also the row max and sum.
    for (int u = 0;; ++u) {
      const int st = u % kStages;
      const bool ok = __all_sync(0xffffffffu, ptx::mbar_wait(ptx::smem_u32(&sm.merged[st]),
                                                             (uint32_t)(u / kStages) & 1, p.status));
      if (!ok) {
        abort_flag = 1;
        break;
      }
      const ItemInfo item = sm.merge_item[st];
      if (item.n < 0) break;
      const float(*mw)[kMergeStride] = sm.merge[st];
      float M = mw[0][kD];
#pragma unroll
      for (int w = 1; w < kConsumerWarps; ++w) M = fmaxf(M, mw[w][kD]);
      float a0 = 0.f, a1 = 0.f, l = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        // warp 0 always has keys, so M is finite and 2^(-inf - M) = 0
        const float s = ptx::ex2_approx(mw[w][kD] - M);
        const float2 a = *reinterpret_cast<const float2 *>(&mw[w][2 * lane]);
        a0 = fmaf(a.x, s, a0);
        a1 = fmaf(a.y, s, a1);
        l = fmaf(mw[w][kD + 1], s, l);
      }
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&sm.merge_free[st]));
      float *part = p.part + ((size_t)item.bh * p.nch + item.c) * kPartFloats;
      *reinterpret_cast<float2 *>(part + 2 * lane) = make_float2(a0, a1);
      if (lane == 0) {
        part[kD] = M;
        part[kD + 1] = l;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g = lane & 7, sub = lane >> 3;  // column group, key within a step
  for (int u = 0;; ++u) {
    const int st = u % kStages;
    const uint32_t par = (uint32_t)(u / kStages) & 1;
    bool ok = __all_sync(0xffffffffu,
                         ptx::mbar_wait(ptx::smem_u32(&sm.full[st]), par, p.status));
    // The merge slot of this stage is free again once its previous use is merged.
    if (ok && u >= kStages)
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(ptx::smem_u32(&sm.merge_free[st]), par ^ 1,
                                                  p.status));
    if (!ok) {
      abort_flag = 1;
      break;
    }
    const ItemInfo item = sm.item[st];
    if (item.n < 0) {
      // Tell the merge warp there is no more work, then stop.
      if (lane == 0) {
        if (warp == 0) sm.merge_item[st].n = -1;
        ptx::mbar_arrive(ptx::smem_u32(&sm.merged[st]));
      }
      break;
    }
    const int n = item.n;

    // Query slice of this lane: columns [8g, 8g+8), pre-scaled.
    constexpr uint32_t kLaneBytes = 8 * sizeof(T);
    float qf[8];
    Elem<T>::load8(sm.q[st] + g * kLaneBytes, qf);
#pragma unroll
    for (int i = 0; i < 8; ++i) qf[i] *= p.scale_log2;

    // ---- scores of this warp's keys t_i = kKeysPerWarp*warp + 4*i + sub (all
    // 8 lanes of a key group end up holding its score).
    const int t_base = kKeysPerWarp * warp + sub;
    const uint8_t *ks = sm.k[st] + g * kLaneBytes;
    float sc[kSteps];
#pragma unroll
    for (int i = 0; i < kSteps; ++i) {
      const int t = t_base + 4 * i;
      float d = 0.f;
      if (t < n) {
        float kf[8];
        Elem<T>::load8(ks + t * kRowBytes, kf);
#pragma unroll
        for (int e = 0; e < 8; ++e) d = fmaf(qf[e], kf[e], d);
      }
      sc[i] = d;
    }
#pragma unroll
    for (int i = 0; i < kSteps; ++i) {
      sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], 1);
      sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], 2);
      sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], 4);
    }
    // ---- warp softmax over its keys
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < kSteps; ++i)
      if (t_base + 4 * i < n) m = fmaxf(m, sc[i]);
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
    float l = 0.f;
#pragma unroll
    for (int i = 0; i < kSteps; ++i) {
      sc[i] = t_base + 4 * i < n ? ptx::ex2_approx(sc[i] - m) : 0.f;
      l += sc[i];
    }
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
    // ---- P.V over the same keys; lane holds columns [8g, 8g+8)
    const uint8_t *vs = sm.v[st] + g * kLaneBytes;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
    for (int i = 0; i < kSteps; ++i) {
      const int t = t_base + 4 * i;
      if (t < n) {
        float vf[8];
        Elem<T>::load8(vs + t * kRowBytes, vf);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(sc[i], vf[e], acc[e]);
      }
    }
    // The stage's K, V and query are no longer read by this warp.
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&sm.empty[st]));
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 8);
      acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 16);
    }
    float *mw = sm.merge[st][warp];
    if (sub == 0) {
      *reinterpret_cast<float4 *>(&mw[8 * g]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4 *>(&mw[8 * g + 4]) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    if (lane == 0) {
      mw[kD] = m;  // -inf for a warp without keys (then l = 0, acc = 0)
      mw[kD + 1] = l;
      if (warp == 0) sm.merge_item[st] = item;
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&sm.merged[st]));
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

// One warp per (batch, head): merge the chunk partials, write f32 output.  The
// partials are independent loads: lane c takes chunk c's (m, l) in one round
// trip, and the column sums issue eight chunks' loads before using any, so a
// row costs a few L2 round trips rather than one per chunk.
template <int kChunk>
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
  for (int c0 = 0; c0 < nc; c0 += 32) {
    // lane i: weight and sum of chunk c0 + i
    const int ci = c0 + lane;
    float w = 0.f;
    if (ci < nc) {
      const float *pc = part + (size_t)ci * kPartFloats;
      const float mc = pc[kD];
      w = mc == -INFINITY ? 0.f : ptx::ex2_approx(mc - M);
      l = fmaf(pc[kD + 1], w, l);
    }
    const int cnt = nc - c0 < 32 ? nc - c0 : 32;
    for (int i = 0; i < cnt; i += 8) {
      float2 a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        a[u] = i + u < cnt ? *reinterpret_cast<const float2 *>(
                                 part + (size_t)(c0 + i + u) * kPartFloats + 2 * lane)
                           : make_float2(0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float wu = __shfl_sync(0xffffffffu, w, (i + u) & 31);
        o0 = fmaf(a[u].x, wu, o0);
        o1 = fmaf(a[u].y, wu, o1);
      }
    }
  }
#pragma unroll
  for (int sh = 16; sh > 0; sh >>= 1) l += __shfl_xor_sync(0xffffffffu, l, sh);
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

bool decode_shape_ok(int64_t B, int64_t H, int64_t max_len) {
  // kv_lens are int32, so a longer cache is never read past 2^31 - 1 rows; the
  // combine kernel's grid covers B*H in blocks of 4 (grid.x < 2^31).
  int64_t bh = 0;
  return B >= 1 && H >= 1 && max_len >= 1 && max_len <= INT32_MAX &&
         !__builtin_mul_overflow(B, H, &bh) && bh <= INT32_MAX;
}

size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t max_len, int64_t, bool f32) {
  // Within decode_shape_ok's bounds: B*H < 2^31 and nch < 2^24, so the
  // partial count stays below 2^55 and the byte count below 2^63.
  if (!decode_shape_ok(B, H, max_len)) return 0;
  const int64_t chunk = f32 ? Chunk<float>::value : Chunk<uint16_t>::value;
  const int64_t nch = (max_len + chunk - 1) / chunk;
  return (size_t)(B * H * nch) * kPartFloats * sizeof(float);
}

namespace {

template <typename T>
cudaError_t launch_decode_t(const DecodeArgs &a, const DeviceInfo &dev, cudaStream_t stream) {
  constexpr int kChunk = Chunk<T>::value;
  if (a.ks.s != kD || a.vs.s != kD) return cudaErrorInvalidValue;  // rows must be contiguous
  if (!decode_shape_ok(a.B, a.H, a.max_len)) return cudaErrorInvalidValue;
  DecParams p;
  p.B = a.B;
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
  const int64_t items = a.B * a.H * p.nch;
  const int64_t blocks = items < dev.sm_count ? items : dev.sm_count;
  static_assert(sizeof(DecSmem<T>) <= 227 * 1024, "shared memory budget");
  const size_t smem = sizeof(DecSmem<T>);
  cudaError_t err = ensure_smem_attr(reinterpret_cast<const void *>(decode_split_kernel<T>),
                                     (int)smem, dev.device);
  if (err != cudaSuccess) return err;
  decode_split_kernel<T><<<(unsigned)blocks, kThreads, smem, stream>>>(p);
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
  decode_combine_kernel<kChunk><<<(unsigned)((cp.BH + 3) / 4), 128, 0, stream>>>(cp);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode(const DecodeArgs &a, const DeviceInfo &dev, cudaStream_t stream) {
  return a.f32 ? launch_decode_t<float>(a, dev, stream) : launch_decode_t<uint16_t>(a, dev, stream);
}

}  // namespace wfattn
