/*
 * wf_oracle.c -- CPU oracle for WarpForth's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links or calls
 * this file.  It is used by tests/ (as the checker), by __graft_entry__.smoke()
 * and by bench.py's CPU-baseline / reference arm.  It is never the thing that
 * is measured as the GPU product.
 *
 * What it restates (file:line are in the reference tree tetsuo-cpp/warpforth):
 *
 *   demo/attention.forth:18-81   the kernel `attention(Q,K,V,O,SEQ_LEN,HEAD_DIM)`
 *     row = BID-X (query row), t = TID-X (key index)
 *     :22-29  s_t = (sum_{i ascending} f64(Q[row,i]) * f64(K[t,i])) / sqrt(f64(D))
 *             F32@ widens f32 -> f64 (lib/Conversion/ForthToMemRef/ForthToMemRef.cpp:854-858),
 *             F* / F+ / F/ are plain f64 arith ops (ForthToMemRef.cpp:508-516),
 *             S>F is sitofp (ForthToMemRef.cpp:1031-1037), FSQRT is math.sqrt (:567).
 *     :31-33  if t > row: s_t = -1.0e30   (finite, not -inf)
 *     :39-45  m = s_0; for I = 1 .. S-1: m = maximumf(m, s_I)  (FMAX = arith.maximumf, :519-520)
 *     :47-52  p_t = exp(s_t - m)                                 (FEXP = math.exp f64, :566)
 *     :54-60  l = 0; for I = 0 .. S-1: l = l + p_I
 *     :62-67  p_t = p_t / l
 *     :69-81  O[row,col] = f32( sum_{j ascending} p_j * f64(V[j,col]) )   (F32! = truncf, :955-960)
 *
 *   The f64 sums are accumulated with separate multiply and add (this file is
 *   compiled with -ffp-contract=off).  Whether the reference's NVPTX backend
 *   contracts them into FMA is unknown; the difference is O(1e-16) relative.
 *
 * Domain: the reference kernel is only valid for 2 <= S <= 1024 (block = S
 * threads; `SEQ_LEN 1 DO` is a post-test loop, lib/Translation/ForthToMLIR/
 * ForthToMLIR.cpp:1081-1085, that does not terminate at S = 1).  The oracle
 * computes the mathematical result for any S >= 1.
 *
 * Generalisation used by the batched entry points (wfo_attention): B x H heads
 * with element strides, Sq queries against Sk keys, an explicit scale (or the
 * reference's divide-by-sqrt(D) when scale <= 0), optional causal masking with
 * the query block aligned to the END of the keys (query i sees keys
 * t <= i + Sk - Sq; identical to the reference when Sq == Sk), and optional
 * per-batch key lengths (decode over a padded KV cache).  Masked keys are
 * skipped instead of being given -1e30: for finite inputs exp(-1e30 - m) is
 * exactly 0.0 in f64, so the sums, the max and the output are bit-identical
 * (tests/test_oracle.py checks this against the literal restatement).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* arith.maximumf: NaN-propagating maximum, and -0.0 < +0.0. */
static double maximumf(double a, double b) {
  if (isnan(a) || isnan(b)) return NAN;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}

/*
 * Literal restatement of demo/attention.forth for one head: Q, K, V, O are
 * contiguous row-major [S, D] arrays.  Loops run over all S keys exactly as
 * the Forth does, including the -1e30 mask value.  `scores` is caller scratch
 * of S doubles (the kernel's `shared SCORES f64[1024]`).  Instantiated for
 * f32 I/O (demo/attention.forth: F32@ / F32!) and for f64 I/O (the test twin
 * gpu_test/test_kernels.py:592-649 and test/Pipeline/attention.forth: F@ / F!).
 */
#define WFO_DEFINE_LITERAL(NAME, T)                                                              \
  static void NAME##_row(const T *Q, const T *K, const T *V, T *O, int64_t S, int64_t D,         \
                         int64_t row, double *scores) {                                          \
    for (int64_t t = 0; t < S; ++t) {                                                            \
      double acc = 0.0;                                                                          \
      for (int64_t i = 0; i < D; ++i) acc = acc + (double)Q[row * D + i] * (double)K[t * D + i]; \
      double s = acc / sqrt((double)D);                                                          \
      if (t > row) s = -1.0e30;                                                                  \
      scores[t] = s;                                                                             \
    }                                                                                            \
    double m = scores[0];                                                                        \
    for (int64_t I = 1; I < S; ++I) m = maximumf(m, scores[I]);                                  \
    for (int64_t t = 0; t < S; ++t) scores[t] = exp(scores[t] - m);                              \
    double l = 0.0;                                                                              \
    for (int64_t I = 0; I < S; ++I) l = l + scores[I];                                           \
    for (int64_t t = 0; t < S; ++t) scores[t] = scores[t] / l;                                   \
    for (int64_t col = 0; col < D; ++col) {                                                      \
      double acc = 0.0;                                                                          \
      for (int64_t j = 0; j < S; ++j) acc = acc + scores[j] * (double)V[j * D + col];            \
      O[row * D + col] = (T)acc;                                                                 \
    }                                                                                            \
  }                                                                                              \
  int NAME(const T *Q, const T *K, const T *V, T *O, int64_t S, int64_t D) {                     \
    if (!Q || !K || !V || !O || S < 1 || D < 1) return 1;                                        \
    double *scores = (double *)malloc((size_t)S * sizeof(double));                               \
    if (!scores) return 2;                                                                       \
    for (int64_t row = 0; row < S; ++row) NAME##_row(Q, K, V, O, S, D, row, scores);             \
    free(scores);                                                                                \
    return 0;                                                                                    \
  }

WFO_DEFINE_LITERAL(wfo_attention_head, float)
WFO_DEFINE_LITERAL(wfo_attention_head_f64, double)

/*
 * One query row of the generalised form.  Same operation order as the
 * literal restatement, restricted to the visible keys [0, nvis).
 */
static void attention_row(const float *q, const float *k, const float *v, float *o, int64_t nvis,
                          int64_t D, int64_t ks, int64_t vs, double scale, int ref_scale,
                          double *p) {
  const double rs = sqrt((double)D);
  for (int64_t t = 0; t < nvis; ++t) {
    const float *kt = k + t * ks;
    double acc = 0.0;
    for (int64_t i = 0; i < D; ++i) acc = acc + (double)q[i] * (double)kt[i];
    p[t] = ref_scale ? acc / rs : acc * scale;
  }
  double m = p[0];
  for (int64_t t = 1; t < nvis; ++t) m = maximumf(m, p[t]);
  for (int64_t t = 0; t < nvis; ++t) p[t] = exp(p[t] - m);
  double l = 0.0;
  for (int64_t t = 0; t < nvis; ++t) l = l + p[t];
  for (int64_t t = 0; t < nvis; ++t) p[t] = p[t] / l;
  for (int64_t col = 0; col < D; ++col) {
    double acc = 0.0;
    for (int64_t j = 0; j < nvis; ++j) acc = acc + p[j] * (double)v[j * vs + col];
    o[col] = (float)acc;
  }
}

/*
 * Batched, strided generalisation.  Strides are in elements, ordered
 * {batch, head, seq}; the head_dim stride is 1.  kv_lens (may be NULL) gives
 * the number of valid keys per batch entry (<= Sk).  Only query rows
 * [row_begin, row_end) of every selected head are computed, and only heads
 * bh in [bh_begin, bh_end) (bh = b*H + h); pass -1 for "all".  nthreads <= 0
 * uses the OpenMP default.  Returns 0 on success.
 */
int wfo_attention(const float *q, const float *k, const float *v, float *o, int64_t B, int64_t H,
                  int64_t Sq, int64_t Sk, int64_t D, const int64_t *qs, const int64_t *ks,
                  const int64_t *vs, const int64_t *os, double scale, int causal,
                  const int32_t *kv_lens, int64_t bh_begin, int64_t bh_end, int64_t row_begin,
                  int64_t row_end, int nthreads) {
  if (!q || !k || !v || !o || !qs || !ks || !vs || !os) return 1;
  if (B < 1 || H < 1 || Sq < 1 || Sk < 1 || D < 1) return 1;
  if (bh_begin < 0) bh_begin = 0;
  if (bh_end < 0 || bh_end > B * H) bh_end = B * H;
  if (row_begin < 0) row_begin = 0;
  if (row_end < 0 || row_end > Sq) row_end = Sq;
  if (bh_begin >= bh_end || row_begin >= row_end) return 0;
  const int ref_scale = !(scale > 0.0);
  const int64_t nrows = row_end - row_begin;
  const int64_t nwork = (bh_end - bh_begin) * nrows;
  int bad = 0;
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads) reduction(| : bad)
#endif
  {
    double *p = (double *)malloc((size_t)Sk * sizeof(double));
    if (!p) {
      bad |= 2;
    } else {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
      for (int64_t w = 0; w < nwork; ++w) {
        const int64_t bh = bh_begin + w / nrows;
        const int64_t i = row_begin + w % nrows;
        const int64_t b = bh / H, h = bh % H;
        int64_t L = kv_lens ? (int64_t)kv_lens[b] : Sk;
        if (L < 1 || L > Sk || (causal && L < Sq)) {
          bad |= 1;
          continue;
        }
        const int64_t nvis = causal ? i + (L - Sq) + 1 : L;
        attention_row(q + b * qs[0] + h * qs[1] + i * qs[2], k + b * ks[0] + h * ks[1],
                      v + b * vs[0] + h * vs[1], o + b * os[0] + h * os[1] + i * os[2], nvis, D,
                      ks[2], vs[2], scale, ref_scale, p);
      }
      free(p);
    }
  }
  return bad;
}

/* Thread count the OpenMP runtime would use by default (for reporting). */
int wfo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
