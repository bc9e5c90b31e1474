// attn_bf16_sm100.cu -- causal flash attention (prefill), bf16 in/out, f32
// accumulation on the 5th-generation tensor cores (tcgen05 + TMEM), K/V
// staged by TMA.  head_dim = 64 (the GPT-2 head shape).
//
// One CTA computes one 128-row query tile of one (batch, head):
//
//   warp 4 (TMA)      Q once, then K_j / V_j 128x64 tiles into a 2-stage ring
//   warp 5 (MMA)      S_j = Q K_j^T         (SS: both operands in smem, K-major)
//                     O  += P_{j-1} V_{j-1} (TS: P from TMEM, V MN-major in smem)
//   warps 0-3         thread r owns query row r: reads S_j from TMEM, online
//                     softmax in the exp2 domain, writes P_j (bf16) to TMEM,
//                     rescales the TMEM O row when its running max moved,
//                     and finally normalises O and stores the bf16 row.
//
// TMEM (256 columns, 2 CTAs per SM): S [0,128)  P [128,192)  O [192,256).
// The MMA warp issues S_{j+1} as soon as the softmax warps have copied S_j
// into registers, and P_j V_j while the softmax warps compute exp2 for
// S_{j+1}, so the tensor core, the MUFU and the FMA pipes overlap; the second
// resident CTA fills the remaining gaps.
//
// Causal tiles above the diagonal are never loaded or multiplied; CTAs are
// issued heaviest-first.  Ragged edges (S not a multiple of 128) rely on TMA
// zero fill plus an explicit key mask.
#include <cuda.h>
#include <math.h>

#include "sm100_ptx.cuh"
#include "tma_map.h"
#include "wfattn_internal.h"

namespace wfattn {
namespace {

constexpr int kBM = 128;           // query rows per CTA (= TMEM lanes)
constexpr int kBN = 128;           // keys per tile
constexpr int kD = 64;             // head_dim
constexpr int kStages = 2;         // K and V ring depth
constexpr int kThreads = 192;      // 4 softmax warps + TMA warp + MMA warp
constexpr uint32_t kTileBytes = kBN * kD * 2;  // 16 KB per 128x64 bf16 tile
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColP = 128, kColO = 192;

struct Smem {
  // 1024-byte aligned tiles (128-byte swizzle atoms)
  uint8_t q[kTileBytes];
  uint8_t k[kStages][kTileBytes];
  uint8_t v[kStages][kTileBytes];
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full, s_free, p_full, o_done;
  uint64_t drain;  // MMA completion barrier used only when aborting
  uint32_t tmem_base;
  uint32_t abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + alignment slack

struct Bf16Params {
  int64_t B, H, Sq, Sk;
  int64_t n_qtiles;
  char *o;
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

__global__ void __launch_bounds__(kThreads, 2)
    prefill_bf16_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const Bf16Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // A timeout recorded by an earlier launch is sticky until the host clears it.
  if (ptx::timeout_flagged(p.status)) return;
  if (threadIdx.x == 0) trace(0, 1);

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
    for (int i = 0; i < kStages; ++i) {
      ptx::mbar_init(ptx::smem_u32(&sm.k_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.k_empty[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.v_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.v_empty[i]), 1);
    }
    ptx::mbar_init(ptx::smem_u32(&sm.s_full), 1);
    ptx::mbar_init(ptx::smem_u32(&sm.s_free), kBM);
    ptx::mbar_init(ptx::smem_u32(&sm.p_full), kBM);
    ptx::mbar_init(ptx::smem_u32(&sm.o_done), 1);
    ptx::mbar_init(ptx::smem_u32(&sm.drain), 1);
    sm.abort = 0;
    ptx::fence_barrier_init();
  }
  if (warp == 4 && lane == 0) {
    ptx::prefetch_tmap(&tm_q);
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_v);
  }
  if (warp == 5) {
    if (lane == 0) trace(1, 1);
    ptx::tmem_alloc(ptx::smem_u32(&sm.tmem_base), kTmemCols);
    ptx::tmem_relinquish();
    if (lane == 0) trace(1, 2);
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  if (threadIdx.x == 0) {
    trace(0, 3);
    trace(7, tmem);
  }

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t qf = ptx::smem_u32(&sm.q_full);
      ptx::mbar_arrive_expect_tx(qf, kTileBytes);
      ptx::tma_load_4d(ptx::smem_u32(sm.q), &tm_q, 0, (int)q0, h, b, qf);
      int issued_k = 0, issued_v = 0;  // loads issued so far (tile index + 1)
      for (int j = 0; j < n_kv && !aborted(sm); ++j) {
        const int st = j % kStages;
        const uint32_t use = (uint32_t)(j / kStages);
        if (j >= kStages &&
            !ptx::mbar_wait(ptx::smem_u32(&sm.k_empty[st]), (use - 1) & 1, p.status)) {
          set_abort(sm);
          break;
        }
        const uint32_t kf = ptx::smem_u32(&sm.k_full[st]);
        ptx::mbar_arrive_expect_tx(kf, kTileBytes);
        ptx::tma_load_4d(ptx::smem_u32(sm.k[st]), &tm_k, 0, j * kBN, h, b, kf);
        issued_k = j + 1;
        if (j >= kStages &&
            !ptx::mbar_wait(ptx::smem_u32(&sm.v_empty[st]), (use - 1) & 1, p.status)) {
          set_abort(sm);
          break;
        }
        const uint32_t vf = ptx::smem_u32(&sm.v_full[st]);
        ptx::mbar_arrive_expect_tx(vf, kTileBytes);
        ptx::tma_load_4d(ptx::smem_u32(sm.v[st]), &tm_v, 0, j * kBN, h, b, vf);
        issued_v = j + 1;
        trace(2, 100 + j);
      }
      trace(2, aborted(sm) ? 6 : 5);
      if (aborted(sm)) {
        // Drain: every load this thread issued must land before the CTA exits.
        ptx::mbar_wait_drain(qf, 0);
        for (int j = imin64(issued_k, kStages) ; j > 0; --j) {
          const int t = issued_k - j;
          ptx::mbar_wait_drain(ptx::smem_u32(&sm.k_full[t % kStages]), (uint32_t)(t / kStages) & 1);
        }
        for (int j = imin64(issued_v, kStages); j > 0; --j) {
          const int t = issued_v - j;
          ptx::mbar_wait_drain(ptx::smem_u32(&sm.v_full[t % kStages]), (uint32_t)(t / kStages) & 1);
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = ptx::idesc_bf16_f32(kBM, kBN, 0, 0);
      constexpr uint32_t idesc_pv = ptx::idesc_bf16_f32(kBM, kD, 0, 1);
      const uint32_t tS = tmem + kColS, tP = tmem + kColP, tO = tmem + kColO;
      const uint32_t q_addr = ptx::smem_u32(sm.q);
      bool ok = ptx::mbar_wait(ptx::smem_u32(&sm.q_full), 0, p.status);
      trace(1, ok ? 3 : 4);

      auto issue_pv = [&](int i) -> bool {
        const int st = i % kStages;
        if (!ptx::mbar_wait(ptx::smem_u32(&sm.p_full), (uint32_t)i & 1, p.status)) return false;
        if (!ptx::mbar_wait(ptx::smem_u32(&sm.v_full[st]), (uint32_t)(i / kStages) & 1, p.status))
          return false;
        ptx::tc_fence_after();
        const uint32_t v_addr = ptx::smem_u32(sm.v[st]);
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          // V as the MN-major B operand: 16 keys = two 8-row swizzle atoms (2 KB).
          const uint64_t bd = ptx::smem_desc_sw128(v_addr + kk * 2048, kTileBytes, 1024);
          ptx::mma_ts(tO, tP + kk * 8, bd, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
        }
        ptx::tc_commit(ptx::smem_u32(&sm.o_done));
        ptx::tc_commit(ptx::smem_u32(&sm.v_empty[st]));
        return true;
      };

      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j % kStages;
        if (!ptx::mbar_wait(ptx::smem_u32(&sm.k_full[st]), (uint32_t)(j / kStages) & 1,
                            p.status)) {
          ok = false;
          break;
        }
        if (j > 0 && !ptx::mbar_wait(ptx::smem_u32(&sm.s_free), (uint32_t)(j - 1) & 1, p.status)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t k_addr = ptx::smem_u32(sm.k[st]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          // K-major operands: advance 16 elements (32 bytes) inside the 128-byte swizzle row.
          const uint64_t ad = ptx::smem_desc_sw128(q_addr + kk * 32, 16, 1024);
          const uint64_t bd = ptx::smem_desc_sw128(k_addr + kk * 32, 16, 1024);
          ptx::mma_ss(tS, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        ptx::tc_commit(ptx::smem_u32(&sm.s_full));
        ptx::tc_commit(ptx::smem_u32(&sm.k_empty[st]));
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) ok = issue_pv(n_kv - 1);
      trace(1, ok ? 5 : 6);
      if (!ok) {
        set_abort(sm);
        // Drain: wait until every MMA this thread issued has completed.
        ptx::tc_commit(ptx::smem_u32(&sm.drain));
        ptx::mbar_wait_drain(ptx::smem_u32(&sm.drain), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0-3
    const int row = threadIdx.x;  // TMEM lane == query row within the tile
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    const int64_t grow = q0 + row;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      // warp-uniform outcome: the tcgen05.ld/st below are warp-collective
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(ptx::smem_u32(&sm.s_full), (uint32_t)j & 1,
                                                  p.status));
      if (!ok) break;
      ptx::tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) ptx::tmem_ld32(lane_base + kColS + c * 32, sr[c]);
      ptx::tmem_wait_ld();
      ptx::tc_fence_before();
      ptx::mbar_arrive(ptx::smem_u32(&sm.s_free));

      const int64_t n0 = (int64_t)j * kBN;
      const bool need_mask = (n0 + kBN > p.Sk) || (p.causal && n0 + kBN - 1 > q0 + off);
      float mx = -INFINITY;
      if (need_mask) {
        const int64_t lim = p.causal ? imin64(grow + off, p.Sk - 1) : p.Sk - 1;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float x = __uint_as_float(sr[c][e]);
            if (n0 + c * 32 + e > lim) x = -INFINITY;
            sr[c][e] = __float_as_uint(x);
            mx = fmaxf(mx, x);
          }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) mx = fmaxf(mx, __uint_as_float(sr[c][e]));
      }
      const float m_new = fmaxf(m_run, mx * p.scale_log2);
      const float alpha = ptx::ex2_approx(m_run - m_new);
      float sum = 0.f;
      uint32_t pk[2][32];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float p0 = ptx::ex2_approx(fmaf(__uint_as_float(sr[c][e]), p.scale_log2, -m_new));
          const float p1 =
              ptx::ex2_approx(fmaf(__uint_as_float(sr[c][e + 1]), p.scale_log2, -m_new));
          sum += p0 + p1;
          pk[c >> 1][(c & 1) * 16 + e / 2] = ptx::pack_bf16x2(p0, p1);
        }
      l_run = l_run * alpha + sum;
      m_run = m_new;

      if (j > 0) {
        // PV_{j-1} must have finished before O is rescaled and P is overwritten.
        ok = __all_sync(0xffffffffu, ptx::mbar_wait(ptx::smem_u32(&sm.o_done),
                                                    (uint32_t)(j - 1) & 1, p.status));
        if (!ok) break;
        ptx::tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            ptx::tmem_ld32(lane_base + kColO + c * 32, o);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            ptx::tmem_st32(lane_base + kColO + c * 32, o);
          }
        }
      }
      ptx::tmem_st32(lane_base + kColP, pk[0]);
      ptx::tmem_st32(lane_base + kColP + 32, pk[1]);
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(ptx::smem_u32(&sm.p_full));
      if (row == 0) trace(3, 100 + j);
    }
    if (ok) {
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(ptx::smem_u32(&sm.o_done),
                                                  (uint32_t)(n_kv - 1) & 1, p.status));
    }
    if (ok) {
      ptx::tc_fence_after();
      const float inv = 1.f / l_run;
      uint32_t o[2][32];
      ptx::tmem_ld32(lane_base + kColO, o[0]);
      ptx::tmem_ld32(lane_base + kColO + 32, o[1]);
      ptx::tmem_wait_ld();
      if (row < qrows) {
        char *dst = p.o + 2 * (b * p.os_b + h * p.os_h + grow * p.os_s);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 w;
          const uint32_t *src = &o[c >> 2][(c & 3) * 8];
          w.x = ptx::pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
          w.y = ptx::pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
          w.z = ptx::pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
          w.w = ptx::pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
          reinterpret_cast<uint4 *>(dst)[c] = w;
        }
      }
    } else {
      set_abort(sm);
    }
  }

  if (threadIdx.x == 0) trace(3, 5);
  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace(6, 1);
  if (warp == 5) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
    if (lane == 0) trace(1, 8);
  }
}

}  // namespace

#ifdef WFATTN_TRACE
cudaError_t set_trace_prefill_1q(void *p) { return set_trace_symbol(p); }
#endif

cudaError_t launch_prefill_bf16_1q(const PrefillArgs &a, const DeviceInfo &dev,
                                   cudaStream_t stream) {
  static_assert(kSmemBytes <= 113 * 1024, "two CTAs per SM must fit");
  CUtensorMap tq, tk, tv;
  if (!make_bf16_map_64x128(&tq, a.q, a.B, a.H, a.Sq, a.qs) ||
      !make_bf16_map_64x128(&tk, a.k, a.B, a.H, a.Sk, a.ks) ||
      !make_bf16_map_64x128(&tv, a.v, a.B, a.H, a.Sk, a.vs))
    return cudaErrorInvalidValue;
  if (a.B > 0x7fffffff || a.H > 0x7fffffff || a.Sk > 0x7fffffff) return cudaErrorInvalidValue;
  cudaError_t err = ensure_smem_attr(reinterpret_cast<const void *>(prefill_bf16_kernel),
                                     (int)kSmemBytes, dev.device);
  if (err != cudaSuccess) return err;
  Bf16Params p;
  p.B = a.B;
  p.H = a.H;
  p.Sq = a.Sq;
  p.Sk = a.Sk;
  p.n_qtiles = (a.Sq + kBM - 1) / kBM;
  p.o = static_cast<char *>(a.o);
  p.os_b = a.os.b;
  p.os_h = a.os.h;
  p.os_s = a.os.s;
  p.scale_log2 = (float)((double)a.scale * 1.4426950408889634);
  p.causal = a.causal;
  p.status = dev.status;
  const int64_t blocks = p.n_qtiles * a.B * a.H;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  prefill_bf16_kernel<<<(unsigned)blocks, kThreads, kSmemBytes, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace wfattn
