// attn_bf16_2q_sm100.cu -- causal flash attention (prefill), bf16 in/out, f32
// accumulation on tcgen05 tensor cores; two 128-row query tiles per CTA.
//
// Persistent: one CTA per SM walks work items of 256 query rows of one
// (batch, head), heaviest first (item_of), each as two 128-row tiles A and B
// that share every K/V tile loaded by TMA (half the L2 -> shared-memory
// traffic per FLOP of one tile per CTA).  All ring and barrier phases are
// counted across items, so the next item's loads and first S overlap the
// current item's tail.
//
//   warp 1 (TMA, K)   Q_A, Q_B of each work item (two slots); K_j tiles into a 3-deep ring
//   warp 2 (TMA, V)   V_j tiles into their own 3-deep ring.  K and V have
//                     separate producers so a K load never waits for a V
//                     slot (V slots free only after P.V, later than K slots).
//   warp 0 (MMA, QK)  S_A(j) = Q_A K_j^T, S_B(j) = Q_B K_j^T, each as soon as
//                     that tile's softmax has read S(j-1) out of TMEM, so the
//                     next scores are computed while the softmax still works
//   warp 3 (MMA, PV)  O_A += P_A(j) V_j, O_B += P_B(j) V_j, each as soon as that
//                     tile's softmax has written P(j)
//   warps 4-7 / 8-11  softmax of tile A / tile B, one query row per thread
//                     (TMEM lane = row, 32x32b loads; warp w reads lanes
//                     32*(w%4)..+31, the sub-partition it may access): the
//                     row max and row sum need no shuffles and each thread
//                     packs its own P row.  At the end of an item each warp
//                     writes its 32 output rows to a staging slab and one
//                     TMA store into the local output; for a fused all-gather
//                     the same lane queues bulk copies of the slab to every
//                     further destination (other GPUs' buffers), so the TMA
//                     engine, not the softmax warp, moves those bytes over
//                     NVLink while the next item computes.  With a multicast
//                     output instead, the warp reads the slab back in 512-byte
//                     runs and writes each 16 bytes once through the multicast
//                     address (multimem.st): the NVLink switch delivers them
//                     to every GPU's buffer, this one's included.
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
//  * kPolyPairsOf8 of every 8 exponential pairs are evaluated on the FMA
//    pipes with the Cody-Waite + minimax polynomial of exp2_poly.cuh
//    (relative error 7.5e-5, below the bf16 rounding of P), the rest on the
//    MUFU ex2 unit, so both run in parallel.  A masked score (-inf) comes
//    out of the polynomial as 2^-126 instead of 0: against the row maximum's
//    p >= 1 that is far below f32 resolution in both the row sum and P.V.
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
constexpr int kSoftmaxWarps = 8;  // 2 tiles x 4 warps of 32 rows
// Helper warps 0-3 (one per scheduler), softmax warps 4-11.
constexpr int kMmaQkWarp = 0, kTmaKWarp = 1, kTmaVWarp = 2, kMmaPvWarp = 3, kFirstSoftmaxWarp = 4;
constexpr int kThreads = 32 * (kSoftmaxWarps + 4);
constexpr uint32_t kTileBytes = kBN * kD * 2;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColP0 = 256, kColO0 = 384;  // tile t: + 128t / 64t / 64t
constexpr float kRescaleLog2 = 8.f;
constexpr int kPolyPairsOf8 = 2;  // exp2 pairs per 8 pairs on the polynomial (25%)

struct Smem {
  uint8_t q[2][2][kTileBytes];  // [slot][tile A/B]: Q of two consecutive work items
  uint8_t k[kStages][kTileBytes];
  uint8_t v[kStages][kTileBytes];
  // Output staging, one 32-row x 128-byte slab per softmax warp (row r at
  // r * 128).  With one destination, 16-byte chunk c of row r sits at chunk
  // c ^ (r % 8) -- the 128-byte swizzle, read by a swizzled TMA tensor store,
  // so that 8 threads writing their rows' chunk c hit 8 different bank groups.
  // With further destinations (which take untiled bulk copies of the rows)
  // the slab is plain row-major for the local TMA store too.
  uint8_t ostage[kSoftmaxWarps][32 * 128];
  uint64_t q_full[2], q_empty[2];
  uint64_t k_full[kStages], k_empty[kStages];
  uint64_t v_full[kStages], v_empty[kStages];
  uint64_t s_full[2], s_free[2], p_full[2], o_done[2], o_free[2];
  uint64_t drain[2];  // per MMA-issuing thread
#ifdef WFATTN_TRACE
  unsigned long long tl[24][64];  // cycle timeline of CTA 0 (trace builds only)
#endif
  uint32_t tmem_base;
  uint32_t abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

struct Params {
  int64_t B, H, Sq, Sk;
  int64_t n_pairs;  // 256-row query blocks per (batch, head)
  int64_t n_items;  // n_pairs * B * H
  uint32_t group;   // consecutive blocks of one (batch, head) in the item order
  // Further destinations of the output (e.g. other GPUs' buffers mapped into
  // this one), written by untiled bulk copies; strides os_* are shared.
  char *remote[kMaxOutputPeers - 1];
  int n_remote;
  // Multicast address of the output (replaces the TMA store and the remote
  // copies when set).
  char *mc;
  int interleave;  // heavy and light rounds alternate (item_of)
  int64_t os_b, os_h, os_s;
  float scale_log2;
  int causal;
  unsigned int *status;
};

// One work item: 256 query rows (tiles A and B) of one (batch, head).
struct Item {
  int b, h;
  int64_t q0;
  int qrows[2], nkv[2], n_kv;
};

// Items are numbered heaviest first (the causal blocks nearest the end of the
// sequence see the most keys), in groups of p.group consecutive 256-row
// blocks of one (batch, head): the group's CTAs run at the same time and
// share that head's K/V tiles in L2 (group 1: every CTA on another head).
// CTA i takes item r*G + i in even rounds r and r*G + (G-1-i) in odd ones
// (G = grid size): the snake order evens out the CTAs' totals.  Returns
// false past the last item.
__device__ __forceinline__ bool item_of(const Params &p, int k, Item &it) {
  // 32-bit arithmetic: the launcher keeps n_items below 2^31.
  const uint32_t G = gridDim.x;
  // Round r of the heaviest-first order holds items r*G .. r*G+G-1.  When the
  // kernel also sends its output to other GPUs, the CTAs take the full rounds
  // alternately from the heavy and the light end (0, F-1, 1, F-2, ...; a
  // partial last round stays last): every item writes the same bytes whatever
  // its length, so in plain order the light items at the end would produce
  // output faster than NVLink takes it.
  uint32_t r = (uint32_t)k;
  const uint32_t F = (uint32_t)p.n_items / G;
  if (p.interleave && r < F) r = (r & 1) ? F - 1 - (r >> 1) : (r >> 1);
  const uint32_t idx = r * G + ((k & 1) ? G - 1 - blockIdx.x : blockIdx.x);
  if ((int64_t)idx >= p.n_items) return false;
  const uint32_t BH = (uint32_t)(p.B * p.H), H = (uint32_t)p.H;
  const uint32_t NP = (uint32_t)p.n_pairs, gs = p.group, n_full = NP / gs;
  uint32_t blk, bh;
  if (idx < n_full * gs * BH) {
    const uint32_t g = idx / (gs * BH), r = idx - g * (gs * BH);
    bh = r / gs;
    blk = g * gs + (r - bh * gs);
  } else {  // the last, partial group
    const uint32_t gl = NP - n_full * gs, r = idx - n_full * gs * BH;
    bh = r / gl;
    blk = n_full * gs + (r - bh * gl);
  }
  const int64_t qp = p.n_pairs - 1 - blk;
  it.b = (int)(bh / H);
  it.h = (int)(bh - (uint32_t)it.b * H);
  it.q0 = qp * 2 * kBM;
  const int64_t off = p.Sk - p.Sq;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int64_t r0 = it.q0 + t * kBM;
    it.qrows[t] = r0 < p.Sq ? (int)imin64(kBM, p.Sq - r0) : 0;
    int64_t kend = p.Sk;
    if (p.causal && it.qrows[t] > 0) kend = imin64(p.Sk, r0 + it.qrows[t] - 1 + off + 1);
    it.nkv[t] = it.qrows[t] > 0 ? (int)((kend + kBN - 1) / kBN) : 0;
  }
  it.n_kv = max(it.nkv[0], it.nkv[1]);
  return true;
}

#ifdef WFATTN_TRACE
#define TL(e, j)                                                  \
  do {                                                            \
    if (blockIdx.x == 0 && (j) < 64) sm.tl[(e)][(j)] = clock64(); \
  } while (0)
#else
#define TL(e, j) \
  do {           \
  } while (0)
#endif

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
                           const __grid_constant__ CUtensorMap tm_v,
                           const __grid_constant__ CUtensorMap tm_o, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (ptx::timeout_flagged(p.status)) return;  // sticky until the host clears it
  if (threadIdx.x == 0) {
    trace(0, 1);
    trace(5, (unsigned int)ptx::globaltimer());  // CTA start (ns, low word)
  }
  const int64_t off = p.Sk - p.Sq;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(ptx::smem_u32(&sm.q_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&sm.q_empty[i]), 1);
    }
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
      ptx::mbar_init(ptx::smem_u32(&sm.o_free[t]), kBM);
    }
    ptx::mbar_init(ptx::smem_u32(&sm.drain[0]), 1);
    ptx::mbar_init(ptx::smem_u32(&sm.drain[1]), 1);
    sm.abort = 0;
    ptx::fence_barrier_init();
    trace(0, 2);
  }
  if (warp == kTmaKWarp && lane == 0) {
    ptx::prefetch_tmap(&tm_q);
    ptx::prefetch_tmap(&tm_k);
  }
  if (warp == kTmaVWarp && lane == 0) {
    ptx::prefetch_tmap(&tm_v);
    ptx::prefetch_tmap(&tm_o);
  }
  if (warp == kMmaQkWarp) {
    if (lane == 0) trace(1, 1);
    ptx::tmem_alloc(ptx::smem_u32(&sm.tmem_base), kTmemCols);
    ptx::tmem_relinquish();
    if (lane == 0) trace(1, 2);
  }
#ifdef WFATTN_TRACE
  for (int i = threadIdx.x; i < 24 * 64; i += kThreads) (&sm.tl[0][0])[i] = 0ull;
#endif
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  if (threadIdx.x == 0) {
    trace(0, 3);
    trace(7, tmem);
  }

  // Every role walks the same item sequence; ring and barrier phases are
  // counted across items, so the next item's loads and S = QK^T overlap the
  // current item's last iterations and its output.
  if (warp == kTmaKWarp || warp == kTmaVWarp) {
    // ------------------------------------------------------------ TMA producers
    if (lane == 0) {
      const bool is_k = warp == kTmaKWarp;
      const CUtensorMap *tm = is_k ? &tm_k : &tm_v;
      uint64_t *full = is_k ? sm.k_full : sm.v_full;
      uint64_t *empty = is_k ? sm.k_empty : sm.v_empty;
      uint8_t(*ring)[kTileBytes] = is_k ? sm.k : sm.v;
      int issued = 0;   // ring loads so far
      int q_items = 0;  // items whose Q was loaded
      bool ok = true;
      Item it;
      for (int k = 0; ok && item_of(p, k, it); ++k) {
        if (is_k) {
          // Q of this item into slot k & 1, once the QKs of item k-2 are done.
          const int slot = k & 1;
          if (k >= 2 && !ptx::mbar_wait(ptx::smem_u32(&sm.q_empty[slot]),
                                        (uint32_t)((k >> 1) - 1) & 1, p.status)) {
            ok = false;
            break;
          }
          const uint32_t qf = ptx::smem_u32(&sm.q_full[slot]);
          const int nq = it.qrows[1] > 0 ? 2 : 1;
          ptx::mbar_arrive_expect_tx(qf, kTileBytes * nq);
          for (int t = 0; t < nq; ++t)
            ptx::tma_load_4d(ptx::smem_u32(sm.q[slot][t]), &tm_q, 0, (int)(it.q0 + t * kBM), it.h,
                             it.b, qf);
          q_items = k + 1;
        }
        for (int j = 0; j < it.n_kv; ++j) {
          const int st = issued % kStages;
          if (aborted(sm) ||
              (issued >= kStages && !ptx::mbar_wait(ptx::smem_u32(&empty[st]),
                                                    (uint32_t)(issued / kStages - 1) & 1,
                                                    p.status))) {
            ok = false;
            break;
          }
          const uint32_t fb = ptx::smem_u32(&full[st]);
          ptx::mbar_arrive_expect_tx(fb, kTileBytes);
          ptx::tma_load_4d(ptx::smem_u32(ring[st]), tm, 0, j * kBN, it.h, it.b, fb);
          if (is_k) TL(20, issued);
          ++issued;
        }
      }
      trace(2, ok ? 5 : 6);
      if (!ok) {
        set_abort(sm);
        // Drain: every load this thread issued must land before the CTA exits.
        for (int i = (int)imin64(q_items, 2); i > 0; --i) {
          const int u = q_items - i;
          ptx::mbar_wait_drain(ptx::smem_u32(&sm.q_full[u & 1]), (uint32_t)(u >> 1) & 1);
        }
        for (int i = (int)imin64(issued, kStages); i > 0; --i) {
          const int u = issued - i;
          ptx::mbar_wait_drain(ptx::smem_u32(&full[u % kStages]), (uint32_t)(u / kStages) & 1);
        }
      }
    }
  } else if (warp == kMmaQkWarp || warp == kMmaPvWarp) {
    // ------------------------------------------------------------ MMA issuers
    // Two threads feed the tensor core: one issues S = Q K^T, the other
    // O += P V.  A tcgen05.mma issue stalls while the tensor pipe is busy, so
    // one thread alone would leave the pipe idle during each of its barrier
    // waits; with two, one waits while the other issues.
    if (lane == 0) {
      const bool is_qk = warp == kMmaQkWarp;
      constexpr uint32_t idesc_qk = ptx::idesc_bf16_f32(kBM, kBN, 0, 0);
      constexpr uint32_t idesc_pv = ptx::idesc_bf16_f32(kBM, kD, 0, 1);
      // Descriptors: constant high halves; low halves = start address >> 4
      // (a K step adds 32 B for Q/K, 2 KB for V; a ring stage or Q tile adds 16 KB).
      const uint64_t dq0 = ptx::smem_desc_sw128(ptx::smem_u32(sm.q[0][0]), 16, 1024);
      const uint64_t dk0 = ptx::smem_desc_sw128(ptx::smem_u32(sm.k[0]), 16, 1024);
      const uint64_t dv0 = ptx::smem_desc_sw128(ptx::smem_u32(sm.v[0]), kTileBytes, 1024);
      const uint32_t hi_qk = (uint32_t)(dk0 >> 32), hi_v = (uint32_t)(dv0 >> 32);
      const uint32_t qlo0 = (uint32_t)dq0, klo0 = (uint32_t)dk0, vlo0 = (uint32_t)dv0;
      constexpr uint32_t kStageLo = kTileBytes >> 4;
      int ring = 0;                 // K (V) tiles consumed so far
      int n_mma[2] = {0, 0};        // S (P.V) products issued per tile half
      int n_items_t[2] = {0, 0};    // items with rows per tile half (P.V thread)
      bool ok = true;
      trace(1, 3);

      Item it;
      for (int k = 0; ok && item_of(p, k, it); ++k) {
        const int slot = k & 1;
        if (is_qk)
          ok = ptx::mbar_wait(ptx::smem_u32(&sm.q_full[slot]), (uint32_t)(k >> 1) & 1, p.status);
        for (int j = 0; ok && j < it.n_kv; ++j, ++ring) {
          const int st = ring % kStages;
          uint64_t *full = is_qk ? sm.k_full : sm.v_full;
          ok = ptx::mbar_wait(ptx::smem_u32(&full[st]), (uint32_t)(ring / kStages) & 1, p.status);
          TL(is_qk ? 18 : 19, ring);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (!ok || j >= it.nkv[t]) continue;
            const int n = n_mma[t];
            if (is_qk) {
              // S_t is free once softmax t has read the previous S_t out of TMEM.
              if (n > 0)
                ok = ptx::mbar_wait(ptx::smem_u32(&sm.s_free[t]), (uint32_t)(n - 1) & 1, p.status);
              if (!ok) continue;
              ptx::tc_fence_after();
              const uint32_t tS = tmem + kColS0 + 128 * t;
              const uint32_t qa = qlo0 + (2 * slot + t) * kStageLo;
              const uint32_t kb = klo0 + st * kStageLo;
              ptx::mma_ss_lh<false>(tS, qa, hi_qk, kb, hi_qk, idesc_qk);
              ptx::mma_ss_lh<true>(tS, qa + 2, hi_qk, kb + 2, hi_qk, idesc_qk);
              ptx::mma_ss_lh<true>(tS, qa + 4, hi_qk, kb + 4, hi_qk, idesc_qk);
              ptx::mma_ss_lh<true>(tS, qa + 6, hi_qk, kb + 6, hi_qk, idesc_qk);
              ptx::tc_commit(ptx::smem_u32(&sm.s_full[t]));
              TL(t, n);
            } else {
              // The first P.V of an item overwrites O_t: softmax t must have
              // read the previous item's O_t.  Every P.V needs P_t written.
              if (j == 0 && n_items_t[t] > 0)
                ok = ptx::mbar_wait(ptx::smem_u32(&sm.o_free[t]),
                                    (uint32_t)(n_items_t[t] - 1) & 1, p.status);
              if (ok)
                ok = ptx::mbar_wait(ptx::smem_u32(&sm.p_full[t]), (uint32_t)n & 1, p.status);
              if (!ok) continue;
              ptx::tc_fence_after();
              const uint32_t tO = tmem + kColO0 + 64 * t, tP = tmem + kColP0 + 64 * t;
              const uint32_t vb = vlo0 + st * kStageLo;
              if (j == 0)
                ptx::mma_ts_lh<false>(tO, tP, vb, hi_v, idesc_pv);
              else
                ptx::mma_ts_lh<true>(tO, tP, vb, hi_v, idesc_pv);
              ptx::mma_ts_lh<true>(tO, tP + 8, vb + 128, hi_v, idesc_pv);
              ptx::mma_ts_lh<true>(tO, tP + 16, vb + 256, hi_v, idesc_pv);
              ptx::mma_ts_lh<true>(tO, tP + 24, vb + 384, hi_v, idesc_pv);
              ptx::mma_ts_lh<true>(tO, tP + 32, vb + 512, hi_v, idesc_pv);
              ptx::mma_ts_lh<true>(tO, tP + 40, vb + 640, hi_v, idesc_pv);
              ptx::mma_ts_lh<true>(tO, tP + 48, vb + 768, hi_v, idesc_pv);
              ptx::mma_ts_lh<true>(tO, tP + 56, vb + 896, hi_v, idesc_pv);
              ptx::tc_commit(ptx::smem_u32(&sm.o_done[t]));
              TL(2 + t, n);
            }
            n_mma[t] = n + 1;
          }
          // Frees the K (V) stage once the MMAs reading it have completed.
          if (ok) ptx::tc_commit(ptx::smem_u32(&(is_qk ? sm.k_empty : sm.v_empty)[st]));
          trace(1, 100 + ring);
        }
        // Frees the Q slot once this item's S products have completed.
        if (ok && is_qk) ptx::tc_commit(ptx::smem_u32(&sm.q_empty[slot]));
#pragma unroll
        for (int t = 0; t < 2; ++t) n_items_t[t] += it.nkv[t] > 0;
      }
      trace(1, ok ? 5 : 6);
      if (!ok) {
        set_abort(sm);
        // Drain: wait until every MMA this thread issued has completed.
        const uint32_t dr = ptx::smem_u32(&sm.drain[is_qk ? 0 : 1]);
        ptx::tc_commit(dr);
        ptx::mbar_wait_drain(dr, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps 4-11
    const int t = (warp - kFirstSoftmaxWarp) >> 2;  // query tile
    const int row = 32 * (warp & 3) + lane;         // TMEM lane == row within the tile
    const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    const uint32_t cS = kColS0 + 128 * t, cP = kColP0 + 64 * t, cO = kColO0 + 64 * t;
    const uint32_t bar_s_full = ptx::smem_u32(&sm.s_full[t]);
    const uint32_t bar_s_free = ptx::smem_u32(&sm.s_free[t]);
    const uint32_t bar_p_full = ptx::smem_u32(&sm.p_full[t]);
    const uint32_t bar_o_done = ptx::smem_u32(&sm.o_done[t]);
    const uint32_t bar_o_free = ptx::smem_u32(&sm.o_free[t]);
    uint8_t *stage = sm.ostage[warp - kFirstSoftmaxWarp];
    const uint64_t c2 = ptx::f2_pack(p.scale_log2, p.scale_log2);
    int ns = 0;  // S tiles of this tile half consumed so far (= P tiles written)
    bool ok = true;
    Item it;
    for (int k = 0; ok && item_of(p, k, it); ++k) {
      const int n = t ? it.nkv[1] : it.nkv[0];
      if (n == 0) continue;  // ragged last block: this half has no rows
      if (lane == 0 && (warp & 3) == (kFirstSoftmaxWarp & 3)) TL(t ? 17 : 11, k);
      const int64_t q_tile = it.q0 + t * kBM;
      const int64_t grow = q_tile + row;  // global query row
      // Key tiles from j_mask on need masking: the ragged last tile (past Sk)
      // and, when causal, the tiles that reach past the tile's first row.
      int j_mask = (int)(p.Sk / kBN);
      if (p.causal) j_mask = (int)imin64(j_mask, (q_tile + off + 1) / kBN);
      const int64_t last_key = p.causal ? imin64(grow + off, p.Sk - 1) : p.Sk - 1;
      float m = -INFINITY;  // running offset of this row (log2 units)
      float l = 0.f;        // running sum of 2^(x - m)
      for (int j = 0; j < n; ++j, ++ns) {
        ok = __all_sync(0xffffffffu, ptx::mbar_wait(bar_s_full, (uint32_t)ns & 1, p.status));
        if (!ok) break;
        ptx::tc_fence_after();
        uint32_t sr[128];
        const bool masked = j >= j_mask;
        // keys c > lim of this tile are masked (lim in [-1, 127] when masked)
        const int lim = masked ? (int)imin64(last_key - (int64_t)j * kBN, 127) : 127;
        float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
        ptx::tmem_ld_32x32b_x64(lane_base + cS, *reinterpret_cast<uint32_t(*)[64]>(&sr[0]));
        ptx::tmem_wait_ld();
        ptx::tmem_ld_32x32b_x64(lane_base + cS + 64, *reinterpret_cast<uint32_t(*)[64]>(&sr[64]));
        // the first half's max overlaps the second half's load
        if (masked) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c > lim) sr[c] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          a0 = ptx::fmax3(a0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
          a1 = ptx::fmax3(a1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
          a2 = ptx::fmax3(a2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
          a3 = ptx::fmax3(a3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
        }
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar_s_free);
        if (lane == 0 && (warp & 3) == (kFirstSoftmaxWarp & 3)) TL(4 + 4 * t, ns);
        if (masked) {
#pragma unroll
          for (int c = 64; c < 128; ++c)
            if (c > lim) sr[c] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int c = 64; c < 128; c += 8) {
          a0 = ptx::fmax3(a0, __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
          a1 = ptx::fmax3(a1, __uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3]));
          a2 = ptx::fmax3(a2, __uint_as_float(sr[c + 4]), __uint_as_float(sr[c + 5]));
          a3 = ptx::fmax3(a3, __uint_as_float(sr[c + 6]), __uint_as_float(sr[c + 7]));
        }
        const float mx = fmaxf(ptx::fmax3(a0, a1, a2), a3) * p.scale_log2;
        float alpha = 1.f;
        if (mx > m + kRescaleLog2) {  // first tile: m = -inf
          alpha = ptx::ex2_approx(m - mx);
          m = mx;
        }
        // P overwrites the previous P of this tile half (possibly the previous
        // item's last): wait until that P.V has completed (which also makes O
        // final for the rescale); P is then stored in 16-column pieces as it
        // is produced.
        if (ns > 0) {
          ok = __all_sync(0xffffffffu,
                          ptx::mbar_wait(bar_o_done, (uint32_t)(ns - 1) & 1, p.status));
          if (!ok) break;
          ptx::tc_fence_after();
        }
        const uint64_t nm = ptx::f2_pack(-m, -m);
        uint64_t s0 = 0, s1 = 0;  // bit pattern 0 == (0.f, 0.f)
        // P row packed in place: pair c reads sr[2c], sr[2c+1] and writes sr[c],
        // which pair c/2 has already read.
        uint32_t(&pk)[64] = *reinterpret_cast<uint32_t(*)[64]>(&sr[0]);
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const uint64_t x2 = ptx::f2_fma(
              ptx::f2_pack(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1])), c2, nm);
          const bool poly = (c & 7) < kPolyPairsOf8;
          const uint64_t p2 = poly ? exp2_poly2(x2) : exp2_mufu2(x2);
          if (c & 1)
            s1 = ptx::f2_add(s1, p2);
          else
            s0 = ptx::f2_add(s0, p2);
          float p0, p1;
          ptx::f2_unpack(p2, p0, p1);
          pk[c] = ptx::pack_bf16x2(p0, p1);
          if ((c & 15) == 15)
            ptx::tmem_st16(lane_base + cP + c - 15,
                           *reinterpret_cast<uint32_t(*)[16]>(&pk[c - 15]));
        }
        {
          float x0, x1;
          ptx::f2_unpack(ptx::f2_add(s0, s1), x0, x1);
          l = l * alpha + (x0 + x1);
        }
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
          uint32_t o[64];
          ptx::tmem_ld_32x32b_x64(lane_base + cO, o);
          ptx::tmem_wait_ld();
          const uint64_t a2 = ptx::f2_pack(alpha, alpha);
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            float w0, w1;
            ptx::f2_unpack(
                ptx::f2_mul(ptx::f2_pack(__uint_as_float(o[c]), __uint_as_float(o[c + 1])), a2),
                w0, w1);
            o[c] = __float_as_uint(w0);
            o[c + 1] = __float_as_uint(w1);
          }
          ptx::tmem_st_32x32b_x64(lane_base + cO, o);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar_p_full);
        if (lane == 0 && (warp & 3) == (kFirstSoftmaxWarp & 3)) TL(12 + 4 * t, ns);
        if (warp == kFirstSoftmaxWarp + 4 * t && lane == 0) trace(3 + t, 100 + ns);
      }
      if (!ok) break;
      // ---- output of this item: O_t / l once the last P.V has completed.
      // O_t is handed back to the P.V thread as soon as it is in registers;
      // the rows go out through this warp's staging slab: one TMA store
      // (rows past Sq are clipped by the tensor map) and, for a fused
      // all-gather, bulk copies of the valid rows to the further destinations.
      ok = __all_sync(0xffffffffu, ptx::mbar_wait(bar_o_done, (uint32_t)(ns - 1) & 1, p.status));
      if (!ok) break;
      if (lane == 0 && (warp & 3) == (kFirstSoftmaxWarp & 3)) TL(t ? 13 : 5, k);
      ptx::tc_fence_after();
      uint32_t o[64];
      ptx::tmem_ld_32x32b_x64(lane_base + cO, o);
      ptx::tmem_wait_ld();
      ptx::tc_fence_before();
      ptx::mbar_arrive(bar_o_free);
      if (lane == 0 && (warp & 3) == (kFirstSoftmaxWarp & 3)) TL(t ? 14 : 6, k);
      const float inv = 1.f / l;
      const uint32_t swz = p.n_remote > 0 ? 0u : (uint32_t)(lane & 7);
      // the previous item's copies must have finished reading the slab
      ptx::bulk_wait_group_read0();
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 w;
        const uint32_t *src = &o[8 * c];
        w.x = ptx::pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
        w.y = ptx::pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
        w.z = ptx::pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
        w.w = ptx::pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
        *reinterpret_cast<uint4 *>(stage + lane * 128 + (((uint32_t)c ^ swz) << 4)) = w;
      }
      ptx::fence_proxy_async_smem();
      __syncwarp();
      const int64_t row0 = q_tile + 32 * (warp & 3);
      if (lane == 0 && p.mc == nullptr)
        ptx::tma_store_4d(&tm_o, ptx::smem_u32(stage), 0, (int)row0, it.h, it.b);
      if (p.mc != nullptr) {
        // Lanes 8i..8i+7 take row 4m+i's 8 chunks in round m (the slab is
        // swizzled: chunk c of row r at c ^ (r % 8)), so each multimem store
        // instruction of the warp covers 4 consecutive rows.
        const int nrows = (int)imin64(32, p.Sq - row0);
        const int64_t head = it.b * p.os_b + it.h * p.os_h;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int r = 4 * m + (lane >> 3), c = lane & 7;
          if (r < nrows) {
            const uint4 w =
                *reinterpret_cast<const uint4 *>(stage + r * 128 + ((c ^ (r & 7)) << 4));
            ptx::multimem_st_v4(p.mc + 2 * (head + (row0 + r) * p.os_s) + 16 * c, w);
          }
        }
      } else if (p.n_remote > 0) {
        // The further destinations (the all-gather of a head-sharded prefill:
        // other GPUs' buffers, written over NVLink) get the slab's valid rows
        // (those below Sq) by untiled bulk copies: one copy per destination
        // when the rows are contiguous there, else one per row, each lane
        // copying its own row.
        const int nrows = (int)imin64(32, p.Sq - row0);
        const int64_t head = it.b * p.os_b + it.h * p.os_h;
        if (p.os_s == kD) {
          if (lane == 0 && nrows > 0) {
            const int64_t off = 2 * (head + row0 * kD);
#pragma unroll
            for (int d = 0; d < kMaxOutputPeers - 1; ++d)
              if (d < p.n_remote)
                ptx::bulk_store(p.remote[d] + off, ptx::smem_u32(stage), (uint32_t)nrows * 128);
          }
        } else if (lane < nrows) {
          const int64_t off = 2 * (head + (row0 + lane) * p.os_s);
#pragma unroll
          for (int d = 0; d < kMaxOutputPeers - 1; ++d)
            if (d < p.n_remote)
              ptx::bulk_store(p.remote[d] + off, ptx::smem_u32(stage + lane * 128), 128);
        }
      }
      ptx::bulk_commit_group();
      if (lane == 0 && (warp & 3) == (kFirstSoftmaxWarp & 3)) TL(t ? 15 : 9, k);
    }
    // Outstanding output copies must complete before the CTA exits.
    ptx::bulk_wait_group0();
    if (p.mc != nullptr) __threadfence_system();  // multicast stores before what follows
    if (!ok) set_abort(sm);
    if (warp == kFirstSoftmaxWarp + 4 * t && lane == 0) trace(3 + t, ok ? 5 : 6);
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    trace(6, 1);
    trace(7, (unsigned int)ptx::globaltimer());  // CTA end (ns, low word)
  }
#ifdef WFATTN_TRACE
  if (blockIdx.x == 0 && g_trace)
    for (int i = threadIdx.x; i < 24 * 64; i += kThreads)
      reinterpret_cast<volatile unsigned long long *>(g_trace + 4096)[i] = (&sm.tl[0][0])[i];
#endif
  if (warp == kMmaQkWarp) {
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
  // The first destination (on this GPU) takes TMA tensor stores of 32-row
  // slabs (128-byte swizzled when it is the only one); the others, untiled
  // bulk copies of the same, then row-major, slabs.
  CUtensorMap to;
  if (a.n_peers > kMaxOutputPeers ||
      !make_bf16_map(&to, a.o_mc ? a.o_mc : a.n_peers > 0 ? a.o_peers[0] : a.o, a.B, a.H, a.Sq,
                     a.os, 64, 32,
                     /*swizzle128=*/a.n_peers <= 1))
    return cudaErrorInvalidValue;
  if (a.B > 0x7fffffff || a.H > 0x7fffffff || a.Sk > 0x7fffffff || a.Sq > 0x7fffffff)
    return cudaErrorInvalidValue;
  cudaError_t err = ensure_smem_attr(reinterpret_cast<const void *>(prefill_bf16_2q_kernel),
                                     (int)kSmemBytes, dev.device);
  if (err != cudaSuccess) return err;
  Params p;
  p.B = a.B;
  p.H = a.H;
  p.Sq = a.Sq;
  p.Sk = a.Sk;
  p.n_pairs = (a.Sq + 2 * kBM - 1) / (2 * kBM);
  p.n_remote = a.n_peers > 1 ? a.n_peers - 1 : 0;
  p.mc = static_cast<char *>(a.o_mc);
  p.interleave = (p.mc != nullptr || p.n_remote > 0) ? 1 : 0;
  if (p.mc && p.n_remote) return cudaErrorInvalidValue;  // one output mode per launch
  for (int d = 0; d < kMaxOutputPeers - 1; ++d)
    p.remote[d] = d < p.n_remote ? static_cast<char *>(a.o_peers[d + 1]) : nullptr;
  p.os_b = a.os.b;
  p.os_h = a.os.h;
  p.os_s = a.os.s;
  p.scale_log2 = (float)((double)a.scale * 1.4426950408889634);
  p.causal = a.causal;
  p.status = dev.status;
  p.n_items = p.n_pairs * a.B * a.H;
  if (p.n_items > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  // Persistent: one CTA per SM walks the items (fewer CTAs for small problems).
  const int64_t blocks = p.n_items < dev.sm_count ? p.n_items : dev.sm_count;
  // Groups of 8 blocks per head cut HBM reads when every CTA has many items
  // (long sequences, 16+ blocks per head); with few items per CTA the plain
  // heaviest-first order balances the CTAs better.
  p.group = (p.n_pairs >= 16 && p.n_items >= 32 * blocks) ? 8 : 1;
  prefill_bf16_2q_kernel<<<(unsigned)blocks, kThreads, kSmemBytes, stream>>>(tq, tk, tv, to, p);
  return cudaGetLastError();
}

}  // namespace wfattn
