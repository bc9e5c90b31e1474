// attn_f32.cu -- f32 flash attention on the CUDA cores of sm_100a.
//
// This is the reference-accurate path: the reference kernel
// (demo/attention.forth:18-81) reads f32, computes in f64 and writes f32.
// Here the whole computation stays in f32 (f32 FMA dot products, online
// softmax with exp2, f32 P.V accumulation), which keeps the output within
// 1e-5 absolute of the f64 reference for the GPT-2 head shapes; the tests
// assert that bound against the CPU oracle.
//
// Shape of the work (one CTA = one query tile of 16*RPT rows of one (batch, head);
// RPT = 8 rows per thread for head_dim <= 64 with more than 64 queries, else 4):
//   for each 64-key tile t visible to the query tile:
//     S = Q K_t^T                 RPT x 4 scores per thread (RPT rows x 4 keys)
//     online softmax per row      row max / sum over the 16 threads of a half warp
//     O += P V_t                  RPT rows x D/16 columns per thread
// The dot products are bound by shared-memory bandwidth (each float4 read
// feeds RPT or 4 FMAs), so the larger RPT of the head_dim-64 tile (8 rows per
// K read) lifts the FMA rate; larger head dims keep RPT = 4 to fit the tile.
// Rows are strided (row i of a thread is ty + 16*i, key j is tx + 16*j) so
// that the shared-memory reads of K and V are conflict free with a +4 float
// row pad.  Causal tiles above the diagonal are never loaded; CTAs are issued
// heaviest-first (last query tile of every head first).
#include <math.h>

#include "wfattn_internal.h"

namespace wfattn {
namespace {

constexpr int kBN = 64;        // keys per tile
constexpr int kThreads = 256;  // 16 x 16

template <int DP, int RPT>
struct F32Layout {
  static constexpr int kBM = 16 * RPT;   // query rows per CTA
  static constexpr int kLd = DP + 4;     // floats per Q/K/V smem row
  static constexpr int kPld = kBN + 16;  // floats per P smem row
  static constexpr size_t kFloats =
      (size_t)kBM * kLd + 2 * (size_t)kBN * kLd + (size_t)kBM * kPld;
  static constexpr size_t kBytes = kFloats * sizeof(float);
};

// Copies `nrows` rows of `D` floats (row stride `stride`) into a [ROWS x DP]
// smem tile with row pitch `ld`, zero-filling the padding.
template <int DP, int ROWS>
__device__ __forceinline__ void load_tile(float *__restrict__ dst, int ld,
                                          const float *__restrict__ src, int64_t stride, int nrows,
                                          int D, bool vec) {
  if (vec) {
    constexpr int kC4 = DP / 4;
    for (int idx = threadIdx.x; idx < ROWS * kC4; idx += kThreads) {
      const int r = idx / kC4, c = (idx % kC4) * 4;
      float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < nrows && c < D) val = __ldg(reinterpret_cast<const float4 *>(src + r * stride + c));
      *reinterpret_cast<float4 *>(dst + r * ld + c) = val;
    }
  } else {
    for (int idx = threadIdx.x; idx < ROWS * DP; idx += kThreads) {
      const int r = idx / DP, c = idx % DP;
      dst[r * ld + c] = (r < nrows && c < D) ? __ldg(src + r * stride + c) : 0.f;
    }
  }
}

template <int DP, int RPT>
__global__ void __launch_bounds__(kThreads, 2)
    prefill_f32_kernel(PrefillArgs a, float scale_log2, int64_t n_qtiles, int vec_in, int vec_out) {
  using L = F32Layout<DP, RPT>;
  constexpr int kBM = L::kBM;
  constexpr int kCpt = DP / 16;  // output columns per thread
  extern __shared__ __align__(16) float smem[];
  float *Qs = smem;
  float *Ks = Qs + kBM * L::kLd;
  float *Vs = Ks + kBN * L::kLd;
  float *Ps = Vs + kBN * L::kLd;

  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t BH = a.B * a.H;
  const int64_t qt = n_qtiles - 1 - (int64_t)blockIdx.x / BH;  // heaviest tiles first
  const int64_t bh = (int64_t)blockIdx.x % BH;
  const int64_t b = bh / a.H, h = bh % a.H;
  const int64_t q0 = qt * kBM;
  const int D = (int)a.D;

  const float *qp = static_cast<const float *>(a.q) + b * a.qs.b + h * a.qs.h + q0 * a.qs.s;
  const float *kp = static_cast<const float *>(a.k) + b * a.ks.b + h * a.ks.h;
  const float *vp = static_cast<const float *>(a.v) + b * a.vs.b + h * a.vs.h;
  float *op = static_cast<float *>(a.o) + b * a.os.b + h * a.os.h + q0 * a.os.s;

  const int qrows = (int)imin64(kBM, a.Sq - q0);
  const int64_t off = a.Sk - a.Sq;  // causal alignment of queries to the end of the keys
  int64_t kend = a.Sk;
  if (a.causal) kend = imin64(a.Sk, q0 + qrows - 1 + off + 1);
  const int nkt = (int)((kend + kBN - 1) / kBN);
  const int d4n = (D + 3) / 4;

  load_tile<DP, kBM>(Qs, L::kLd, qp, a.qs.s, qrows, D, vec_in);

  float m[RPT], l[RPT], acc[RPT][kCpt];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < kCpt; ++c) acc[i][c] = 0.f;
  }

  for (int kt = 0; kt < nkt; ++kt) {
    const int64_t n0 = (int64_t)kt * kBN;
    const int krows = (int)imin64(kBN, a.Sk - n0);
    __syncthreads();  // previous tile's K/V/P reads are done
    load_tile<DP, kBN>(Ks, L::kLd, kp + n0 * a.ks.s, a.ks.s, krows, D, vec_in);
    load_tile<DP, kBN>(Vs, L::kLd, vp + n0 * a.vs.s, a.vs.s, krows, D, vec_in);
    __syncthreads();

    float s[RPT][4];
#pragma unroll
    for (int i = 0; i < RPT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;

#pragma unroll 1
    for (int d4 = 0; d4 < d4n; ++d4) {
      float4 kb[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        kb[j] = *reinterpret_cast<const float4 *>(Ks + (tx + 16 * j) * L::kLd + d4 * 4);
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const float4 qa = *reinterpret_cast<const float4 *>(Qs + (ty + 16 * i) * L::kLd + d4 * 4);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qa.x, kb[j].x, s[i][j]);
          s[i][j] = fmaf(qa.y, kb[j].y, s[i][j]);
          s[i][j] = fmaf(qa.z, kb[j].z, s[i][j]);
          s[i][j] = fmaf(qa.w, kb[j].w, s[i][j]);
        }
      }
    }

    const bool need_mask = (n0 + kBN > a.Sk) || (a.causal && n0 + kBN - 1 > q0 + off);
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int64_t row = q0 + ty + 16 * i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float x = s[i][j] * scale_log2;
        if (need_mask) {
          const int64_t key = n0 + tx + 16 * j;
          if (key >= a.Sk || (a.causal && key > row + off)) x = -INFINITY;
        }
        s[i][j] = x;
        mx = fmaxf(mx, x);
      }
#pragma unroll
      for (int sh = 1; sh < 16; sh <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, sh));
      const float m_new = fmaxf(m[i], mx);  // finite: key 0 of tile 0 is visible to every row
      const float alpha = exp2f(m[i] - m_new);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = exp2f(s[i][j] - m_new);
        rs += p;
        Ps[(ty + 16 * i) * L::kPld + tx + 16 * j] = p;
      }
#pragma unroll
      for (int sh = 1; sh < 16; sh <<= 1) rs += __shfl_xor_sync(0xffffffffu, rs, sh);
      l[i] = l[i] * alpha + rs;
      m[i] = m_new;
#pragma unroll
      for (int c = 0; c < kCpt; ++c) acc[i][c] *= alpha;
    }
    __syncthreads();

    const int n4n = (krows + 3) / 4;
    if constexpr (kCpt == 4) {
      // head_dim <= 64: the four V rows of a key group first (16 registers),
      // then one P float4 per row, so few values are live at once.
#pragma unroll 2
      for (int n4 = 0; n4 < n4n; ++n4) {
        float4 vb[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          vb[u] = *reinterpret_cast<const float4 *>(Vs + (n4 * 4 + u) * L::kLd + tx * 4);
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const float4 pa = *reinterpret_cast<const float4 *>(Ps + (ty + 16 * i) * L::kPld + n4 * 4);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float p = u == 0 ? pa.x : u == 1 ? pa.y : u == 2 ? pa.z : pa.w;
            acc[i][0] = fmaf(p, vb[u].x, acc[i][0]);
            acc[i][1] = fmaf(p, vb[u].y, acc[i][1]);
            acc[i][2] = fmaf(p, vb[u].z, acc[i][2]);
            acc[i][3] = fmaf(p, vb[u].w, acc[i][3]);
          }
        }
      }
    } else {
#pragma unroll 2
      for (int n4 = 0; n4 < n4n; ++n4) {
        float4 pa[RPT];
#pragma unroll
        for (int i = 0; i < RPT; ++i)
          pa[i] = *reinterpret_cast<const float4 *>(Ps + (ty + 16 * i) * L::kPld + n4 * 4);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float *vrow = Vs + (n4 * 4 + u) * L::kLd;
#pragma unroll
          for (int kk = 0; kk < kCpt / 4; ++kk) {
            const float4 vb = *reinterpret_cast<const float4 *>(vrow + (tx + 16 * kk) * 4);
#pragma unroll
            for (int i = 0; i < RPT; ++i) {
              const float p = u == 0 ? pa[i].x : u == 1 ? pa[i].y : u == 2 ? pa[i].z : pa[i].w;
              acc[i][kk * 4 + 0] = fmaf(p, vb.x, acc[i][kk * 4 + 0]);
              acc[i][kk * 4 + 1] = fmaf(p, vb.y, acc[i][kk * 4 + 1]);
              acc[i][kk * 4 + 2] = fmaf(p, vb.z, acc[i][kk * 4 + 2]);
              acc[i][kk * 4 + 3] = fmaf(p, vb.w, acc[i][kk * 4 + 3]);
            }
          }
        }
      }
    }
  }

#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = ty + 16 * i;
    if (r >= qrows) continue;
    const float inv = 1.f / l[i];
    float *orow = op + r * a.os.s;
#pragma unroll
    for (int kk = 0; kk < kCpt / 4; ++kk) {
      const int c = (tx + 16 * kk) * 4;
      if (c >= D) continue;
      const float4 val = make_float4(acc[i][kk * 4 + 0] * inv, acc[i][kk * 4 + 1] * inv,
                                     acc[i][kk * 4 + 2] * inv, acc[i][kk * 4 + 3] * inv);
      if (vec_out) {
        *reinterpret_cast<float4 *>(orow + c) = val;
      } else {
        orow[c] = val.x;
        if (c + 1 < D) orow[c + 1] = val.y;
        if (c + 2 < D) orow[c + 2] = val.z;
        if (c + 3 < D) orow[c + 3] = val.w;
      }
    }
  }
}

template <int DP, int RPT>
cudaError_t launch_dp(const PrefillArgs &a, int device, cudaStream_t stream) {
  using L = F32Layout<DP, RPT>;
  static_assert(L::kBytes <= 227 * 1024, "f32 tile does not fit in shared memory");
  cudaError_t err = ensure_smem_attr(reinterpret_cast<const void *>(prefill_f32_kernel<DP, RPT>),
                                     (int)L::kBytes, device);
  if (err != cudaSuccess) return err;
  const int64_t n_qtiles = (a.Sq + L::kBM - 1) / L::kBM;
  const int64_t blocks = n_qtiles * a.B * a.H;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;

  auto aligned16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec_in = (a.D % 4 == 0) && aligned16(a.q) && aligned16(a.k) && aligned16(a.v) &&
                      a.qs.b % 4 == 0 && a.qs.h % 4 == 0 && a.qs.s % 4 == 0 && a.ks.b % 4 == 0 &&
                      a.ks.h % 4 == 0 && a.ks.s % 4 == 0 && a.vs.b % 4 == 0 && a.vs.h % 4 == 0 &&
                      a.vs.s % 4 == 0;
  const bool vec_out = (a.D % 4 == 0) && aligned16(a.o) && a.os.b % 4 == 0 && a.os.h % 4 == 0 &&
                       a.os.s % 4 == 0;
  const double log2e = 1.4426950408889634;
  const float scale_log2 = (float)((double)a.scale * log2e);
  prefill_f32_kernel<DP, RPT><<<(unsigned)blocks, kThreads, L::kBytes, stream>>>(
      a, scale_log2, n_qtiles, vec_in ? 1 : 0, vec_out ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_prefill_f32(const PrefillArgs &a, const DeviceInfo &dev, cudaStream_t stream) {
  // 128-row tiles for head_dim <= 64 unless the queries fit one 64-row tile
  // (short sequences such as the per-token GPT-2 calls would be half padding).
  if (a.D <= 64) return a.Sq > 64 ? launch_dp<64, 8>(a, dev.device, stream)
                                  : launch_dp<64, 4>(a, dev.device, stream);
  if (a.D <= 128) return launch_dp<128, 4>(a, dev.device, stream);
  return launch_dp<256, 4>(a, dev.device, stream);
}

}  // namespace wfattn
