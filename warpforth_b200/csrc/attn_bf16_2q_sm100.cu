// attn_bf16_2q_sm100.cu -- causal flash attention (prefill), bf16 in/out, f32
// accumulation on tcgen05 tensor cores; two 128-row query tiles per CTA.
//
// One CTA (one per SM) computes 256 query rows of one (batch, head) as two
// 128-row tiles A and B that share every K/V tile loaded by TMA, which halves
// the L2 -> shared-memory traffic per FLOP compared with one tile per CTA.
//
//   warp 8 (TMA)     Q_A, Q_B once; then K_j, V_j 128x64 tiles into a ring
//   warp 9 (MMA)     S_A = Q_A K_j^T, S_B = Q_B K_j^T        (SS form)
//                    O_A += P_A V_{j-1}, O_B += P_B V_{j-1}  (TS form, P from TMEM)
//   warps 0-3 / 4-7  softmax of tile A / tile B: thread r owns query row r,
//                    reads S from TMEM, writes bf16 P to TMEM, rescales its O
//                    row in TMEM when needed, and stores the normalised row.
//
// TMEM (512 columns): S_A [0,128) S_B [128,256) P_A [256,320) P_B [320,384)
//                     O_A [384,448) O_B [448,512).
//
// Softmax details (per row, exp2 domain, x = s * scale * log2(e)):
//  * the running offset m only moves when the tile maximum exceeds it by more
//    than kRescaleLog2 (= 8): p = 2^(x - m) <= 256 stays exact enough in
//    bf16/f32, and O / l are rescaled (by 2^(m_old - m_new)) only on those
//    rare steps;
//  * scale-and-subtract, sums and rescales use packed f32x2 FMA/ADD/MUL, the
//    row max uses the three-input max;
//  * kPolyPairsOf8 of every 8 exponential pairs are evaluated on the FMA pipes with the
//    Cody-Waite + minimax polynomial of exp2_poly.cuh (relative error 7.5e-5,
//    below the bf16 rounding of P), the rest on the MUFU ex2 unit; the two
//    units then run in parallel.  Masked (diagonal / ragged) tiles use MUFU
//    only.
#include <cuda.h>
#include <math.h>

#include "exp2_poly.cuh"
#include "sm100_ptx.cuh"
#include "tma_map.h"
#include "wfattn_internal.h"

namespace wfattn {
namespace {

constexpr int kBM = 128;  // rows per query tile (= TMEM lanes)
constexpr int kBN = 128;  // keys per K/V tile
constexpr int kD = 64;
constexpr int kStages = 3;
constexpr int kThreads = 320;  // 8 softmax warps + TMA warp + MMA warp
constexpr uint32_t kTileBytes = kBN * kD * 2;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColP0 = 256, kColO0 = 384;  // tile t: + 128t / 64t / 64t
constexpr float kRescaleLog2 = 8.f;
constexpr int kPolyPairsOf8 = 3;  // exp2 pairs per 8 pairs on the polynomial (37.5%)

struct Smem {
  uint8_t q[2][kTileBytes];
  uint8_t k[kStages][kTileBytes];
  uint8_t v[kStages][kTileBytes];
  uint64_t q_full;
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full[2], s_free[2], p_full[2], o_done[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

struct Params {
  int64_t B, H, Sq, Sk;
  int64_t n_pairs;  // 256-row query blocks per (batch, head)
  char *o;
  int64_t os_b, os_h, os_s;
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

// 2^x for a pair of x, on the FMA pipes: x = j + r, j = round(x), r in [-1/2, 1/2];
// 2^r by the minimax cubic, 2^j added to the exponent field.  x is clamped to
// -126 first: then j >= -126 and 2^r >= 2^-1/2 keeps the biased exponent field
// >= 0, so it never wraps (2^-126 is ~0 against the row maximum p >= 1).
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
  float x0, x1;
  ptx::f2_unpack(x2, x0, x1);
  x2 = ptx::f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t magic = ptx::f2_pack(12582912.f, 12582912.f);  // 1.5 * 2^23
  const uint64_t t = ptx::f2_add(x2, magic);                    // round(x) in the low bits
  const uint64_t j = ptx::f2_add(t, ptx::f2_pack(-12582912.f, -12582912.f));
  const uint64_t r = ptx::f2_fma(j, ptx::f2_pack(-1.f, -1.f), x2);
  uint64_t p = ptx::f2_fma(ptx::f2_pack(exp2poly::kC3, exp2poly::kC3), r,
                           ptx::f2_pack(exp2poly::kC2, exp2poly::kC2));
  p = ptx::f2_fma(p, r, ptx::f2_pack(exp2poly::kC1, exp2poly::kC1));
  p = ptx::f2_fma(p, r, ptx::f2_pack(exp2poly::kC0, exp2poly::kC0));
  float p0, p1, t0, t1;
  ptx::f2_unpack(p, p0, p1);
  ptx::f2_unpack(t, t0, t1);
  // (bits(t) << 23) == j << 23 modulo 2^32 because bits(1.5 * 2^23) << 23 wraps to 0.
  p0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
  return ptx::f2_pack(p0, p1);
}

__device__ __forceinline__ uint64_t exp2_mufu2(uint64_t x2) {
  float x0, x1;
  ptx::f2_unpack(x2, x0, x1);
  return ptx::f2_pack(ptx::ex2_approx(x0), ptx::ex2_approx(x1));
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_bf16_2q_kernel(const __grid_constant__ CUtensorMap tm_q,
                           const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (ptx::timeout_flagged(p.status)) return;  // sticky until the host clears it
  if (threadIdx.x == 0) trace(0, 1);

  const int64_t BH = p.B * p.H;
  const int64_t qp = p.n_pairs - 1 - (int64_t)blockIdx.x / BH;  // heaviest first
  const int64_t bh = (int64_t)blockIdx.x % BH;
  const int b = (int)(bh / p.H), h = (int)(bh % p.H);
  const int64_t q0 = qp * 2 * kBM;
  const int64_t off = p.Sk - p.Sq;
  int qrows[2], nkv[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int64_t r0 = q0 + t * kBM;
    qrows[t] = r0 < p.Sq ? (int)imin64(kBM, p.Sq - r0) : 0;
    int64_t kend = p.Sk;
    if (p.causal && qrows[t] > 0) kend = imin64(p.Sk, r0 + qrows[t] - 1 + off + 1);
    nkv[t] = qrows[t] > 0 ? (int)((kend + kBN - 1) / kBN) : 0;
  }
  const int n_kv = max(nkv[0], nkv[1]);

  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(&sm.q_full), 1);
    for (int i = 0; i < kStages; ++i) {
      ptx::mbar_init(ptx::smem_u32(&sm.k_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.k_empty[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.v_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.v_empty[i]), 1);
    }
    for (int t = 0; t < 2; ++t) {
      ptx::mbar_init(ptx::smem_u32(&sm.s_full[t]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.s_free[t]), kBM);
      ptx::mbar_init(ptx::smem_u32(&sm.p_full[t]), kBM);
      ptx::mbar_init(ptx::smem_u32(&sm.o_done[t]), 1);
    }
    ptx::mbar_init(ptx::smem_u32(&sm.drain), 1);
    sm.abort = 0;
    ptx::fence_barrier_init();
    trace(0, 2);
  }
  if (warp == 8 && lane == 0) {
    ptx::prefetch_tmap(&tm_q);
    ptx::prefetch_tmap(&tm_k);
    ptx::prefetch_tmap(&tm_v);
  }
  if (warp == 9) {
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

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint32_t qf = ptx::smem_u32(&sm.q_full);
      const int nq = qrows[1] > 0 ? 2 : 1;
      ptx::mbar_arrive_expect_tx(qf, kTileBytes * nq);
      for (int t = 0; t < nq; ++t)
        ptx::tma_load_4d(ptx::smem_u32(sm.q[t]), &tm_q, 0, (int)(q0 + t * kBM), h, b, qf);
      trace(2, 1);
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
        ptx::mbar_wait_drain(qf, 0);
        for (int i = (int)imin64(issued_k, kStages); i > 0; --i) {
          const int t = issued_k - i;
          ptx::mbar_wait_drain(ptx::smem_u32(&sm.k_full[t % kStages]), (uint32_t)(t / kStages) & 1);
        }
        for (int i = (int)imin64(issued_v, kStages); i > 0; --i) {
          const int t = issued_v - i;
          ptx::mbar_wait_drain(ptx::smem_u32(&sm.v_full[t % kStages]), (uint32_t)(t / kStages) & 1);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = ptx::idesc_bf16_f32(kBM, kBN, 0, 0);
      constexpr uint32_t idesc_pv = ptx::idesc_bf16_f32(kBM, kD, 0, 1);
      bool ok = ptx::mbar_wait(ptx::smem_u32(&sm.q_full), 0, p.status);
      trace(1, ok ? 3 : 4);

      auto issue_pv = [&](int i) -> bool {
        const int st = i % kStages;
        if (!ptx::mbar_wait(ptx::smem_u32(&sm.v_full[st]), (uint32_t)(i / kStages) & 1, p.status))
          return false;
        const uint32_t v_addr = ptx::smem_u32(sm.v[st]);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (i >= nkv[t]) continue;
          if (!ptx::mbar_wait(ptx::smem_u32(&sm.p_full[t]), (uint32_t)i & 1, p.status))
            return false;
          ptx::tc_fence_after();
          const uint32_t tO = tmem + kColO0 + 64 * t, tP = tmem + kColP0 + 64 * t;
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint64_t bd = ptx::smem_desc_sw128(v_addr + kk * 2048, kTileBytes, 1024);
            ptx::mma_ts(tO, tP + kk * 8, bd, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
          }
          ptx::tc_commit(ptx::smem_u32(&sm.o_done[t]));
        }
        ptx::tc_commit(ptx::smem_u32(&sm.v_empty[st]));
        trace(1, 10000 + i);
        return true;
      };

      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j % kStages;
        if (!ptx::mbar_wait(ptx::smem_u32(&sm.k_full[st]), (uint32_t)(j / kStages) & 1,
                            p.status)) {
          ok = false;
          break;
        }
        const uint32_t k_addr = ptx::smem_u32(sm.k[st]);
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (j >= nkv[t]) continue;
          if (j > 0 &&
              !ptx::mbar_wait(ptx::smem_u32(&sm.s_free[t]), (uint32_t)(j - 1) & 1, p.status)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t q_addr = ptx::smem_u32(sm.q[t]);
          const uint32_t tS = tmem + kColS0 + 128 * t;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint64_t ad = ptx::smem_desc_sw128(q_addr + kk * 32, 16, 1024);
            const uint64_t bd = ptx::smem_desc_sw128(k_addr + kk * 32, 16, 1024);
            ptx::mma_ss(tS, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          ptx::tc_commit(ptx::smem_u32(&sm.s_full[t]));
        }
        if (!ok) break;
        ptx::tc_commit(ptx::smem_u32(&sm.k_empty[st]));
        trace(1, 100 + j);
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) ok = issue_pv(n_kv - 1);
      trace(1, ok ? 5 : 6);
      if (!ok) {
        set_abort(sm);
        ptx::tc_commit(ptx::smem_u32(&sm.drain));
        ptx::mbar_wait_drain(ptx::smem_u32(&sm.drain), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0-7
    const int t = warp >> 2;             // query tile of this warpgroup
    const int row = threadIdx.x & 127;   // TMEM lane == row within the tile
    const int n = nkv[t];
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t cS = kColS0 + 128 * t, cP = kColP0 + 64 * t, cO = kColO0 + 64 * t;
    const int64_t grow = q0 + t * kBM + row;
    const uint32_t bar_s_full = ptx::smem_u32(&sm.s_full[t]);
    const uint32_t bar_s_free = ptx::smem_u32(&sm.s_free[t]);
    const uint32_t bar_p_full = ptx::smem_u32(&sm.p_full[t]);
    const uint32_t bar_o_done = ptx::smem_u32(&sm.o_done[t]);
    const uint64_t c2 = ptx::f2_pack(p.scale_log2, p.scale_log2);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = n > 0;
    for (int j = 0; j < n; ++j) {
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(bar_s_full, (uint32_t)j & 1, p.status));
      if (!ok) break;
      ptx::tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) ptx::tmem_ld32(lane_base + cS + c * 32, sr[c]);
      ptx::tmem_wait_ld();
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar_s_free);

      const int64_t n0 = (int64_t)j * kBN;
      const bool masked = (n0 + kBN > p.Sk) || (p.causal && n0 + kBN - 1 > q0 + t * kBM + off);
      if (masked) {
        const int64_t lim = p.causal ? imin64(grow + off, p.Sk - 1) : p.Sk - 1;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (n0 + c * 32 + e > lim) sr[c][e] = __float_as_uint(-INFINITY);
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          mx0 = ptx::fmax3(mx0, __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
          mx1 = ptx::fmax3(mx1, __uint_as_float(sr[c][e + 2]), __uint_as_float(sr[c][e + 3]));
          mx2 = ptx::fmax3(mx2, __uint_as_float(sr[c][e + 4]), __uint_as_float(sr[c][e + 5]));
          mx3 = ptx::fmax3(mx3, __uint_as_float(sr[c][e + 6]), __uint_as_float(sr[c][e + 7]));
        }
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * p.scale_log2;
      float alpha = 1.f;
      if (mx > m_run + kRescaleLog2) {  // first tile: m_run = -inf
        alpha = ptx::ex2_approx(m_run - mx);
        m_run = mx;
      }
      const uint64_t nm2 = ptx::f2_pack(-m_run, -m_run);
      uint64_t sum2a = 0, sum2b = 0;  // bit pattern 0 == (0.f, 0.f)
      uint32_t pk[2][32];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const uint64_t s2 = ptx::f2_pack(__uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
          const uint64_t x2 = ptx::f2_fma(s2, c2, nm2);
          const bool poly = !masked && (((e & 15) >> 1) < kPolyPairsOf8);
          const uint64_t p2 = poly ? exp2_poly2(x2) : exp2_mufu2(x2);
          if (e & 2)
            sum2b = ptx::f2_add(sum2b, p2);
          else
            sum2a = ptx::f2_add(sum2a, p2);
          float p0, p1;
          ptx::f2_unpack(p2, p0, p1);
          pk[c >> 1][(c & 1) * 16 + e / 2] = ptx::pack_bf16x2(p0, p1);
        }
      float sa0, sa1, sb0, sb1;
      ptx::f2_unpack(sum2a, sa0, sa1);
      ptx::f2_unpack(sum2b, sb0, sb1);
      l_run = l_run * alpha + ((sa0 + sa1) + (sb0 + sb1));

      if (j > 0) {
        ok = __all_sync(0xffffffffu, ptx::mbar_wait(bar_o_done, (uint32_t)(j - 1) & 1, p.status));
        if (!ok) break;
        ptx::tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          const uint64_t a2 = ptx::f2_pack(alpha, alpha);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t o[32];
            ptx::tmem_ld32(lane_base + cO + c * 32, o);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const uint64_t v2 = ptx::f2_mul(
                  ptx::f2_pack(__uint_as_float(o[e]), __uint_as_float(o[e + 1])), a2);
              float v0, v1;
              ptx::f2_unpack(v2, v0, v1);
              o[e] = __float_as_uint(v0);
              o[e + 1] = __float_as_uint(v1);
            }
            ptx::tmem_st32(lane_base + cO + c * 32, o);
          }
        }
      }
      ptx::tmem_st32(lane_base + cP, pk[0]);
      ptx::tmem_st32(lane_base + cP + 32, pk[1]);
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar_p_full);
      if (row == 0) trace(3 + t, 100 + j);
    }
    if (ok) ok = __all_sync(0xffffffffu, ptx::mbar_wait(bar_o_done, (uint32_t)(n - 1) & 1, p.status));
    if (ok) {
      ptx::tc_fence_after();
      const float inv = 1.f / l_run;
      uint32_t o[2][32];
      ptx::tmem_ld32(lane_base + cO, o[0]);
      ptx::tmem_ld32(lane_base + cO + 32, o[1]);
      ptx::tmem_wait_ld();
      if (row < qrows[t]) {
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
    } else if (n > 0) {
      set_abort(sm);
    }
    if (row == 0) trace(3 + t, ok ? 5 : 6);
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) trace(6, 1);
  if (warp == 9) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
    if (lane == 0) trace(1, 8);
  }
}

}  // namespace

#ifdef WFATTN_TRACE
cudaError_t set_trace_prefill_2q(void *p) { return set_trace_symbol(p); }
#endif

cudaError_t launch_prefill_bf16_2q(const PrefillArgs &a, const DeviceInfo &dev,
                                   cudaStream_t stream) {
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  CUtensorMap tq, tk, tv;
  if (!make_bf16_map_64x128(&tq, a.q, a.B, a.H, a.Sq, a.qs) ||
      !make_bf16_map_64x128(&tk, a.k, a.B, a.H, a.Sk, a.ks) ||
      !make_bf16_map_64x128(&tv, a.v, a.B, a.H, a.Sk, a.vs))
    return cudaErrorInvalidValue;
  if (a.B > 0x7fffffff || a.H > 0x7fffffff || a.Sk > 0x7fffffff || a.Sq > 0x7fffffff)
    return cudaErrorInvalidValue;
  cudaError_t err = cudaFuncSetAttribute(
      prefill_bf16_2q_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
  if (err != cudaSuccess) return err;
  Params p;
  p.B = a.B;
  p.H = a.H;
  p.Sq = a.Sq;
  p.Sk = a.Sk;
  p.n_pairs = (a.Sq + 2 * kBM - 1) / (2 * kBM);
  p.o = static_cast<char *>(a.o);
  p.os_b = a.os.b;
  p.os_h = a.os.h;
  p.os_s = a.os.s;
  p.scale_log2 = (float)((double)a.scale * 1.4426950408889634);
  p.causal = a.causal;
  p.status = dev.status;
  const int64_t blocks = p.n_pairs * a.B * a.H;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  prefill_bf16_2q_kernel<<<(unsigned)blocks, kThreads, kSmemBytes, stream>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace wfattn
