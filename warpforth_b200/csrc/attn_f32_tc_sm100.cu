// attn_f32_tc_sm100.cu -- f32 flash attention (prefill) on the tcgen05 tensor
// cores, for head_dim 64: the reference-accurate path (f32 in and out, within
// 1e-5 absolute of the reference kernel's f64 arithmetic) at tensor-core rate.
//
// Precision: every f32 operand x is split into hi + lo, where hi is x with
// the 13 low mantissa bits dropped (what a kind::tf32 MMA reads from an f32
// bit pattern) and lo = x - hi (exact in f32).  Each product is formed from
// three tf32 MMAs, a_hi*b_hi + a_hi*b_lo + a_lo*b_hi, accumulated in f32 (the
// dropped lo*lo term is below 2^-20 of the product): the "3xTF32" split.  The
// softmax is f32 (ex2.approx, relative error ~2^-22), P stays f32 and is split
// the same way for P.V.
//
// One CTA computes one 128-row query tile of one (batch, head), heaviest
// tiles first; keys in 64-key steps.
//   warp 4      TMA: Q (two 128-byte-wide column halves) once, K_j and V_j
//               (each two halves of 64 rows) into 2-stage rings
//   warps 6-9   the lo parts: Q once, then K_j of every stage, each thread
//               writing its share of a tile at the same swizzled byte offsets;
//               V_j is transposed on the way (V^T hi and lo, K-major with the
//               keys contiguous), so that every tf32 operand is K-major; then a
//               proxy fence and arrival
//   warp 5      S(j) = Q K_j^T: 3 x 8 MMAs (N = 64 keys) into S/P buffer j % 2
//   warp 10     O += P(j) V_j: 3 x 8 MMAs (N = 64 = head_dim), P from TMEM
//   warps 0-3   softmax, one query row per thread: S from TMEM, online
//               softmax in the exp2 domain, P (f32) written over S and its lo
//               part next to it; O rescaled only when the running maximum
//               moves by more than 2^8; finally O / l stored as f32 rows.
// TMEM: S/P buffer b at 128 b (P over S's 64 columns, P's lo at +64); O at 256.
// QK^T(j) reuses buffer j % 2 once P.V(j - 2) has completed.
#include <cuda.h>
#include <math.h>

#include "sm100_ptx.cuh"
#include "tma_map.h"
#include "wfattn_internal.h"

namespace wfattn {
namespace {

constexpr int kBM = 128;  // query rows per CTA (= TMEM lanes)
constexpr int kBN = 64;   // keys per step
constexpr int kD = 64;
constexpr int kStages = 2;
constexpr int kThreads = 32 * 11;
constexpr int kTmaWarp = 4, kQkWarp = 5, kFirstSplitWarp = 6, kPvWarp = 10;
constexpr int kSplitThreads = 128;
constexpr uint32_t kQHalf = kBM * 128;  // 16 KB: 128 rows x 32 floats
constexpr uint32_t kKvHalf = kBN * 128;  // 8 KB: 64 rows x 32 floats
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColBuf = 128, kColPlo = 64, kColO = 256;
constexpr float kRescaleLog2 = 8.f;

struct Smem {
  uint8_t q[2][2][kQHalf];             // [hi/lo][column half]
  uint8_t k[kStages][2][2][kKvHalf];   // [stage][hi/lo][column half]
  // [stage][as loaded ([key][dim]) / V^T hi / V^T lo ([dim][key])][half]
  uint8_t v[kStages][3][2][kKvHalf];
  uint64_t q_full, q_lo;
  uint64_t k_full[kStages], k_lo[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_lo[kStages], v_empty[kStages];
  uint64_t s_full[2], p_full[2], pv_done[2];
  uint64_t drain[2];
  uint32_t tmem_base;
  uint32_t abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

struct TcParams {
  int64_t B, H, Sq, Sk;
  int64_t n_qtiles;
  float *o;
  int64_t os_b, os_h, os_s;  // element strides
  float scale_log2;
  int causal;
  unsigned int *status;
};

__device__ __forceinline__ bool aborted(const Smem &s) {
  return *reinterpret_cast<const volatile uint32_t *>(&s.abort) != 0;
}
__device__ __forceinline__ void set_abort(Smem &s) {
  *reinterpret_cast<volatile uint32_t *>(&s.abort) = 1;
}

// x with the 13 low mantissa bits dropped: the tf32 value an MMA reads.
__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xffffe000u);
}

// Writes lo = x - hi(x) of `bytes` of f32 data at src into dst (same offsets).
__device__ __forceinline__ void split_lo(const uint8_t *src, uint8_t *dst, uint32_t bytes,
                                         int tid) {
  for (uint32_t i = (uint32_t)tid * 16; i < bytes; i += kSplitThreads * 16) {
    float4 x = *reinterpret_cast<const float4 *>(src + i);
    x.x -= tf32_hi(x.x);
    x.y -= tf32_hi(x.y);
    x.z -= tf32_hi(x.z);
    x.w -= tf32_hi(x.w);
    *reinterpret_cast<float4 *>(dst + i) = x;
  }
}

// Byte offset of element (r, c) of a tile of 128-byte rows (32 floats) in
// halves of kKvHalf bytes by column block of 32, 128-byte swizzle (16-byte
// chunk index xor row % 8) -- the layout TMA writes and the MMA reads.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)(c >> 5) * kKvHalf + (uint32_t)r * 128 +
         ((uint32_t)(((c & 31) >> 2) ^ (r & 7)) << 4) + (uint32_t)(c & 3) * 4;
}

// V_j as loaded (row = key, 64 dims) -> V_j^T hi and lo (row = dim, 64 keys),
// 4 x 4 blocks per thread.  16-byte accesses are served 8 threads at a time;
// the 8 threads t of group g take key quad 8 (g & 1) + t and dim quad
// 8 ((g >> 1) & 1) + (t ^ (g >> 2)) -- a diagonal, so their loads (rows = keys)
// and their transposed stores (rows = dims) each fall on the 8 distinct
// swizzle chunk positions (bank groups) of a 128-byte row: no bank conflicts.
__device__ __forceinline__ void transpose_split_v(const uint8_t *v, uint8_t *vt_hi,
                                                  uint8_t *vt_lo, int tid) {
  for (int blk = tid; blk < 256; blk += kSplitThreads) {
    const int g = blk >> 3, t = blk & 7;
    const int k0 = 4 * (8 * (g & 1) + t), d0 = 4 * (8 * ((g >> 1) & 1) + (t ^ (g >> 2)));
    float4 r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = *reinterpret_cast<const float4 *>(v + sw128_off(k0 + i, d0));
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      const float a0 = d == 0 ? r[0].x : d == 1 ? r[0].y : d == 2 ? r[0].z : r[0].w;
      const float a1 = d == 0 ? r[1].x : d == 1 ? r[1].y : d == 2 ? r[1].z : r[1].w;
      const float a2 = d == 0 ? r[2].x : d == 1 ? r[2].y : d == 2 ? r[2].z : r[2].w;
      const float a3 = d == 0 ? r[3].x : d == 1 ? r[3].y : d == 2 ? r[3].z : r[3].w;
      const uint32_t o = sw128_off(d0 + d, k0);
      *reinterpret_cast<float4 *>(vt_hi + o) = make_float4(a0, a1, a2, a3);
      *reinterpret_cast<float4 *>(vt_lo + o) =
          make_float4(a0 - tf32_hi(a0), a1 - tf32_hi(a1), a2 - tf32_hi(a2), a3 - tf32_hi(a3));
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_f32_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (ptx::timeout_flagged(p.status)) return;  // sticky until the host clears it

  const int64_t BH = p.B * p.H;
  const int64_t qt = p.n_qtiles - 1 - (int64_t)blockIdx.x / BH;  // heaviest first
  const int64_t bh = (int64_t)blockIdx.x % BH;
  const int b = (int)(bh / p.H), h = (int)(bh % p.H);
  const int64_t q0 = qt * kBM;
  const int qrows = (int)imin64(kBM, p.Sq - q0);
  const int64_t off = p.Sk - p.Sq;
  int64_t kend = p.Sk;
  if (p.causal) kend = imin64(p.Sk, q0 + qrows - 1 + off + 1);
  const int n_kv = (int)((kend + kBN - 1) / kBN);

  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(&sm.q_full), 1);
    ptx::mbar_init(ptx::smem_u32(&sm.q_lo), kSplitThreads);
    for (int i = 0; i < kStages; ++i) {
      ptx::mbar_init(ptx::smem_u32(&sm.k_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.k_lo[i]), kSplitThreads);
      ptx::mbar_init(ptx::smem_u32(&sm.k_empty[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.v_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.v_lo[i]), kSplitThreads);
      ptx::mbar_init(ptx::smem_u32(&sm.v_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(ptx::smem_u32(&sm.s_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.p_full[i]), kBM);
      ptx::mbar_init(ptx::smem_u32(&sm.pv_done[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.drain[i]), 1);
    }
    sm.abort = 0;
    ptx::fence_barrier_init();
  }
  if (warp == kTmaWarp && lane == 0) {
    ptx::prefetch_tmap(&tm_q);
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_v);
  }
  if (warp == kQkWarp) {
    ptx::tmem_alloc(ptx::smem_u32(&sm.tmem_base), kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == kTmaWarp) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t qf = ptx::smem_u32(&sm.q_full);
      ptx::mbar_arrive_expect_tx(qf, 2 * kQHalf);
      for (int c = 0; c < 2; ++c)
        ptx::tma_load_4d(ptx::smem_u32(sm.q[0][c]), &tm_q, 32 * c, (int)q0, h, b, qf);
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < n_kv && !aborted(sm); ++j) {
        const int st = j % kStages;
        const uint32_t use = (uint32_t)(j / kStages);
        if (j >= kStages &&
            !ptx::mbar_wait(ptx::smem_u32(&sm.k_empty[st]), (use - 1) & 1, p.status)) {
          set_abort(sm);
          break;
        }
        const uint32_t kf = ptx::smem_u32(&sm.k_full[st]);
        ptx::mbar_arrive_expect_tx(kf, 2 * kKvHalf);
        for (int c = 0; c < 2; ++c)
          ptx::tma_load_4d(ptx::smem_u32(sm.k[st][0][c]), &tm_k, 32 * c, j * kBN, h, b, kf);
        issued_k = j + 1;
        if (j >= kStages &&
            !ptx::mbar_wait(ptx::smem_u32(&sm.v_empty[st]), (use - 1) & 1, p.status)) {
          set_abort(sm);
          break;
        }
        const uint32_t vf = ptx::smem_u32(&sm.v_full[st]);
        ptx::mbar_arrive_expect_tx(vf, 2 * kKvHalf);
        for (int c = 0; c < 2; ++c)
          ptx::tma_load_4d(ptx::smem_u32(sm.v[st][0][c]), &tm_v, 32 * c, j * kBN, h, b, vf);
        issued_v = j + 1;
      }
      if (aborted(sm)) {
        // Drain: every load this thread issued must land before the CTA exits.
        ptx::mbar_wait_drain(qf, 0);
        for (int i = (int)imin64(issued_k, kStages); i > 0; --i) {
          const int u = issued_k - i;
          ptx::mbar_wait_drain(ptx::smem_u32(&sm.k_full[u % kStages]), (uint32_t)(u / kStages) & 1);
        }
        for (int i = (int)imin64(issued_v, kStages); i > 0; --i) {
          const int u = issued_v - i;
          ptx::mbar_wait_drain(ptx::smem_u32(&sm.v_full[u % kStages]), (uint32_t)(u / kStages) & 1);
        }
      }
    }
  } else if (warp >= kFirstSplitWarp && warp < kFirstSplitWarp + 4) {
    // ------------------------------------------------------------ lo parts
    const int tid = threadIdx.x - 32 * kFirstSplitWarp;
    bool ok = ptx::mbar_wait(ptx::smem_u32(&sm.q_full), 0, p.status);
    if (ok) {
      split_lo(sm.q[0][0], sm.q[1][0], 2 * kQHalf, tid);  // both column halves
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(ptx::smem_u32(&sm.q_lo));
    }
    for (int j = 0; ok && j < n_kv; ++j) {
      const int st = j % kStages;
      const uint32_t par = (uint32_t)(j / kStages) & 1;
      ok = ptx::mbar_wait(ptx::smem_u32(&sm.k_full[st]), par, p.status);
      if (!ok) break;
      split_lo(sm.k[st][0][0], sm.k[st][1][0], 2 * kKvHalf, tid);
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(ptx::smem_u32(&sm.k_lo[st]));
      ok = ptx::mbar_wait(ptx::smem_u32(&sm.v_full[st]), par, p.status);
      if (!ok) break;
      transpose_split_v(sm.v[st][0][0], sm.v[st][1][0], sm.v[st][2][0], tid);
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(ptx::smem_u32(&sm.v_lo[st]));
    }
    if (!ok) set_abort(sm);
  } else if (warp == kQkWarp || warp == kPvWarp) {
    // ------------------------------------------------------------ MMA issuers
    if (lane == 0) {
      const bool is_qk = warp == kQkWarp;
      bool ok = true;
      if (is_qk) {
        constexpr uint32_t idesc = ptx::idesc_tf32_f32(kBM, kBN, 0, 0);
        ok = ptx::mbar_wait(ptx::smem_u32(&sm.q_full), 0, p.status) &&
             ptx::mbar_wait(ptx::smem_u32(&sm.q_lo), 0, p.status);
        for (int j = 0; ok && j < n_kv; ++j) {
          const int st = j % kStages, bf = j & 1;
          const uint32_t par = (uint32_t)(j / kStages) & 1;
          ok = ptx::mbar_wait(ptx::smem_u32(&sm.k_full[st]), par, p.status) &&
               ptx::mbar_wait(ptx::smem_u32(&sm.k_lo[st]), par, p.status);
          // S/P buffer bf is free once P.V(j - 2) has read its P.
          if (ok && j >= 2)
            ok = ptx::mbar_wait(ptx::smem_u32(&sm.pv_done[bf]), (uint32_t)((j - 2) >> 1) & 1,
                                p.status);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint32_t tS = tmem + kColBuf * bf;
#pragma unroll
          for (int kk = 0; kk < kD / 8; ++kk) {
            // K-major operands: 8 floats (32 bytes) per step inside a 128-byte row;
            // columns 32-63 live in the second half.
            const int c = kk >> 2;
            const uint32_t o32 = (uint32_t)(kk & 3) * 32;
            const uint64_t qh = ptx::smem_desc_sw128(ptx::smem_u32(sm.q[0][c]) + o32, 16, 1024);
            const uint64_t ql = ptx::smem_desc_sw128(ptx::smem_u32(sm.q[1][c]) + o32, 16, 1024);
            const uint64_t kh = ptx::smem_desc_sw128(ptx::smem_u32(sm.k[st][0][c]) + o32, 16, 1024);
            const uint64_t kl = ptx::smem_desc_sw128(ptx::smem_u32(sm.k[st][1][c]) + o32, 16, 1024);
            ptx::mma_tf32_ss(tS, qh, kh, idesc, kk > 0 ? 1u : 0u);
            ptx::mma_tf32_ss(tS, qh, kl, idesc, 1u);
            ptx::mma_tf32_ss(tS, ql, kh, idesc, 1u);
          }
          ptx::tc_commit(ptx::smem_u32(&sm.s_full[bf]));
          ptx::tc_commit(ptx::smem_u32(&sm.k_empty[st]));
        }
      } else {
        constexpr uint32_t idesc = ptx::idesc_tf32_f32(kBM, kD, 0, 0);
        const uint32_t tO = tmem + kColO;
        for (int j = 0; ok && j < n_kv; ++j) {
          const int st = j % kStages, bf = j & 1;
          const uint32_t par = (uint32_t)(j / kStages) & 1;
          ok = ptx::mbar_wait(ptx::smem_u32(&sm.v_full[st]), par, p.status) &&
               ptx::mbar_wait(ptx::smem_u32(&sm.v_lo[st]), par, p.status) &&
               ptx::mbar_wait(ptx::smem_u32(&sm.p_full[bf]), (uint32_t)(j >> 1) & 1, p.status);
          if (!ok) break;
          ptx::tc_fence_after();
          const uint32_t tP = tmem + kColBuf * bf;
#pragma unroll
          for (int kk = 0; kk < kBN / 8; ++kk) {
            // V^T as the K-major B operand: 8 keys (32 bytes) per step inside a
            // 128-byte row; keys 32-63 live in the second half.
            const int c = kk >> 2;
            const uint32_t o32 = (uint32_t)(kk & 3) * 32;
            const uint64_t vh = ptx::smem_desc_sw128(ptx::smem_u32(sm.v[st][1][c]) + o32, 16, 1024);
            const uint64_t vl = ptx::smem_desc_sw128(ptx::smem_u32(sm.v[st][2][c]) + o32, 16, 1024);
            const uint32_t ph = tP + kk * 8, pl = tP + kColPlo + kk * 8;
            ptx::mma_tf32_ts(tO, ph, vh, idesc, (j > 0 || kk > 0) ? 1u : 0u);
            ptx::mma_tf32_ts(tO, ph, vl, idesc, 1u);
            ptx::mma_tf32_ts(tO, pl, vh, idesc, 1u);
          }
          ptx::tc_commit(ptx::smem_u32(&sm.pv_done[bf]));
          ptx::tc_commit(ptx::smem_u32(&sm.v_empty[st]));
        }
      }
      if (!ok) {
        set_abort(sm);
        // Drain: wait until every MMA this thread issued has completed.
        const uint32_t dr = ptx::smem_u32(&sm.drain[is_qk ? 0 : 1]);
        ptx::tc_commit(dr);
        ptx::mbar_wait_drain(dr, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0-3
    const int row = threadIdx.x;  // TMEM lane == query row within the tile
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const int64_t grow = q0 + row;
    const int64_t lim_row = p.causal ? imin64(grow + off, p.Sk - 1) : p.Sk - 1;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int bf = j & 1;
      const uint32_t cS = kColBuf * bf;
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(ptx::smem_u32(&sm.s_full[bf]),
                                                  (uint32_t)(j >> 1) & 1, p.status));
      if (!ok) break;
      ptx::tc_fence_after();
      uint32_t sr[64];
      ptx::tmem_ld_32x32b_x64(lane_base + cS, sr);
      ptx::tmem_wait_ld();
      const int64_t n0 = (int64_t)j * kBN;
      if (n0 + kBN - 1 > lim_row) {
        const int64_t lim = lim_row - n0;  // keys c > lim are masked
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c > lim) sr[c] = __float_as_uint(-INFINITY);
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; c += 2)
        mx = ptx::fmax3(mx, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
      mx *= p.scale_log2;
      float alpha = 1.f;
      if (mx > m + kRescaleLog2) {  // first step: m = -inf
        alpha = ptx::ex2_approx(m - mx);
        m = mx;
      }
      float sum = 0.f;
      uint32_t plo[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float pv = ptx::ex2_approx(fmaf(__uint_as_float(sr[c]), p.scale_log2, -m));
        sum += pv;
        sr[c] = __float_as_uint(pv);  // P over S
        plo[c] = __float_as_uint(pv - tf32_hi(pv));
      }
      ptx::tmem_st_32x32b_x64(lane_base + cS, sr);
      ptx::tmem_st_32x32b_x64(lane_base + cS + kColPlo, plo);
      l = l * alpha + sum;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // O must be final: P.V(j - 1) (and every earlier one) has completed.
        ok = __all_sync(0xffffffffu, ptx::mbar_wait(ptx::smem_u32(&sm.pv_done[(j - 1) & 1]),
                                                    (uint32_t)((j - 1) >> 1) & 1, p.status));
        if (!ok) break;
        ptx::tc_fence_after();
        uint32_t o[64];
        ptx::tmem_ld_32x32b_x64(lane_base + kColO, o);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 64; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
        ptx::tmem_st_32x32b_x64(lane_base + kColO, o);
      }
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(ptx::smem_u32(&sm.p_full[bf]));
    }
    if (ok)
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(ptx::smem_u32(&sm.pv_done[(n_kv - 1) & 1]),
                                                  (uint32_t)((n_kv - 1) >> 1) & 1, p.status));
    if (ok) {
      ptx::tc_fence_after();
      uint32_t o[64];
      ptx::tmem_ld_32x32b_x64(lane_base + kColO, o);
      ptx::tmem_wait_ld();
      if (row < qrows) {
        const float inv = 1.f / l;
        float *dst = p.o + b * p.os_b + h * p.os_h + grow * p.os_s;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          reinterpret_cast<float4 *>(dst)[c] = make_float4(
              __uint_as_float(o[4 * c]) * inv, __uint_as_float(o[4 * c + 1]) * inv,
              __uint_as_float(o[4 * c + 2]) * inv, __uint_as_float(o[4 * c + 3]) * inv);
      }
    } else {
      set_abort(sm);
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kQkWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

bool prefill_f32_tc_supported(const PrefillArgs &a) {
  auto al16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  const Strides3 *all[4] = {&a.qs, &a.ks, &a.vs, &a.os};
  for (const Strides3 *x : all)
    if (x->b % 4 || x->h % 4 || x->s % 4) return false;  // 16-byte rows for TMA / float4
  const int64_t ext_q[3] = {a.B, a.H, a.Sq}, ext_k[3] = {a.B, a.H, a.Sk};
  const int64_t sq[3] = {a.qs.b, a.qs.h, a.qs.s}, sk[3] = {a.ks.b, a.ks.h, a.ks.s},
                sv[3] = {a.vs.b, a.vs.h, a.vs.s};
  for (int i = 0; i < 3; ++i)
    if ((ext_q[i] > 1 && sq[i] == 0) || (ext_k[i] > 1 && (sk[i] == 0 || sv[i] == 0)))
      return false;  // broadcast strides: not for TMA
  return a.D == kD && al16(a.q) && al16(a.k) && al16(a.v) && al16(a.o) && a.B <= 0x7fffffff &&
         a.H <= 0x7fffffff && a.Sq <= 0x7fffffff && a.Sk <= 0x7fffffff;
}

cudaError_t launch_prefill_f32_tc(const PrefillArgs &a, const DeviceInfo &dev,
                                  cudaStream_t stream) {
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  CUtensorMap tq, tk, tv;
  if (!make_f32_map(&tq, a.q, a.B, a.H, a.Sq, a.qs, kBM) ||
      !make_f32_map(&tk, a.k, a.B, a.H, a.Sk, a.ks, kBN) ||
      !make_f32_map(&tv, a.v, a.B, a.H, a.Sk, a.vs, kBN))
    return cudaErrorInvalidValue;
  cudaError_t err = ensure_smem_attr(reinterpret_cast<const void *>(prefill_f32_tc_kernel),
                                     (int)kSmemBytes, dev.device);
  if (err != cudaSuccess) return err;
  TcParams p;
  p.B = a.B;
  p.H = a.H;
  p.Sq = a.Sq;
  p.Sk = a.Sk;
  p.n_qtiles = (a.Sq + kBM - 1) / kBM;
  p.o = static_cast<float *>(a.o);
  p.os_b = a.os.b;
  p.os_h = a.os.h;
  p.os_s = a.os.s;
  p.scale_log2 = (float)((double)a.scale * 1.4426950408889634);
  p.causal = a.causal;
  p.status = dev.status;
  const int64_t blocks = p.n_qtiles * a.B * a.H;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  prefill_f32_tc_kernel<<<(unsigned)blocks, kThreads, kSmemBytes, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace wfattn
