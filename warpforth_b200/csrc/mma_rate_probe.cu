// mma_rate_probe.cu -- measures how many SM cycles one tcgen05.mma instruction
// takes when a single thread issues them back to back, for the shapes the
// prefill kernels use (M = 128 rows, K = 16, bf16 operands, f32 accumulation):
//   QK^T  SS form, N = 128 keys        (attn_bf16_2q_sm100.cu, S = Q K^T)
//   P.V   TS form, N = 64 = head_dim   (P from TMEM, V from shared memory)
// and, for comparison, SS N = 256 / N = 64, several independent accumulators,
// a 1:2 mix of the two kernel shapes, and the same streams split over two or
// four issuing threads (one per warp, each into its own accumulator).  One CTA
// per SM, every CTA runs the same streams; operands are zero (the rate does
// not depend on the values).
// Every TMEM column and shared-memory byte addressed lies inside the CTA's
// own allocation (512 TMEM columns, 64 KB of operands); the completion wait is
// bounded by 1 s of %globaltimer.
//
// Usage: wfattn-mma-probe   (prints one line per case)
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "sm100_ptx.cuh"

namespace wfattn {
namespace {

constexpr int kIssued = 256;  // MMAs per timed stream

struct __align__(1024) ProbeSmem {
  uint8_t a[16384];  // 128 x 64 bf16, 128-byte swizzle (Q or A operand)
  uint8_t b[32768];  // 256 x 64 bf16 (K / B operand, up to N = 256)
  uint8_t v[16384];  // 128 x 64 bf16, read MN-major (V)
  uint64_t bar;
  uint32_t tmem;
};

enum Case { kQk, kN256, kN64, kPv, kMix, kQk2, kQk4, kPv2, kQkIss2, kQkIss4, kPvIss2, kPvIss4,
            kMixIss4, kCases };
const char *kNames[kCases] = {"SS N=128 (QK^T)", "SS N=256", "SS N=64", "TS N=64 (P.V)",
                              "QK^T : P.V 1:2", "SS N=128, 2 accum.", "SS N=128, 4 accum.",
                              "TS N=64, 2 accum.", "SS N=128, 2 issuers", "SS N=128, 4 issuers",
                              "TS N=64, 2 issuers", "TS N=64, 4 issuers",
                              "QK^T:P.V 1:2, 2 issuers"};

constexpr double kQkF = 2.0 * 128 * 128 * 16, kPvF = 2.0 * 128 * 64 * 16;
const double kFlop[kCases] = {kQkF, 2.0 * 128 * 256 * 16, kPvF, kPvF, (kQkF + 2 * kPvF) / 3,
                              kQkF, kQkF, kPvF, kQkF, kQkF, kPvF, kPvF, (kQkF + 2 * kPvF) / 3};

__constant__ int kIssuersDev[kCases] = {1, 1, 1, 1, 1, 1, 1, 1, 2, 4, 2, 4, 2};

__global__ void __launch_bounds__(128, 1) mma_rate_kernel(int which, unsigned long long *out) {
  extern __shared__ uint8_t raw[];
  ProbeSmem &sm = *reinterpret_cast<ProbeSmem *>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                                 ~uintptr_t(1023));
  constexpr int kVec = (int)((sizeof(sm.a) + sizeof(sm.b) + sizeof(sm.v)) / 16);
  for (int i = threadIdx.x; i < kVec; i += blockDim.x)
    reinterpret_cast<uint4 *>(sm.a)[i] = make_uint4(0, 0, 0, 0);
  const int issuers = kIssuersDev[which];
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(&sm.bar), (uint32_t)issuers);
    ptx::fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    ptx::tmem_alloc(ptx::smem_u32(&sm.tmem), 512);
    ptx::tmem_relinquish();
  }
  ptx::fence_proxy_async_smem();
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sm.tmem;
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0 && warp < issuers) {
    const uint64_t da = ptx::smem_desc_sw128(ptx::smem_u32(sm.a), 16, 1024);
    const uint64_t db = ptx::smem_desc_sw128(ptx::smem_u32(sm.b), 16, 1024);
    const uint64_t dv = ptx::smem_desc_sw128(ptx::smem_u32(sm.v), 16384, 1024);
    const uint32_t hi = (uint32_t)(da >> 32), hv = (uint32_t)(dv >> 32);
    const uint32_t alo = (uint32_t)da, blo = (uint32_t)db, vlo = (uint32_t)dv;
    constexpr uint32_t i128 = ptx::idesc_bf16_f32(128, 128, 0, 0);
    constexpr uint32_t i256 = ptx::idesc_bf16_f32(128, 256, 0, 0);
    constexpr uint32_t i64 = ptx::idesc_bf16_f32(128, 64, 0, 0);
    constexpr uint32_t ipv = ptx::idesc_bf16_f32(128, 64, 0, 1);
    // TMEM: accumulators in columns [0, 256) (N = 256 uses all of them) and
    // [384, 512); P (the TS form's A operand) in [256, 320).
    // issuer w takes every issuers-th MMA of the stream, into its own accumulator:
    // SS columns [128 w, 128 w + 128), TS columns [64 w, 64 w + 64) (P stays in [256, 320))
    const uint32_t own_ss = tmem + (uint32_t)warp * 128, own_ts = tmem + (uint32_t)warp * 64;
    const long long t0 = clock64();
    for (int i = warp; i < kIssued; i += issuers) {
      const uint32_t k = (uint32_t)(i & 3) * 2;        // K step: 32 bytes along the swizzled row
      const uint32_t kp = (uint32_t)(i & 7);           // P.V K step: 16 keys
      const uint32_t pa = tmem + 256 + kp * 8, vb = vlo + kp * 128;
      switch (which) {
        case kQk: ptx::mma_ss_lh<true>(tmem, alo + k, hi, blo + k, hi, i128); break;
        case kN256: ptx::mma_ss_lh<true>(tmem, alo + k, hi, blo + k, hi, i256); break;
        case kN64: ptx::mma_ss_lh<true>(tmem, alo + k, hi, blo + k, hi, i64); break;
        case kPv: ptx::mma_ts_lh<true>(tmem + 384, pa, vb, hv, ipv); break;
        case kMix:
          if (i % 3 == 0)
            ptx::mma_ss_lh<true>(tmem, alo + k, hi, blo + k, hi, i128);
          else
            ptx::mma_ts_lh<true>(tmem + 384, pa, vb, hv, ipv);
          break;
        case kQk2: ptx::mma_ss_lh<true>(tmem + (uint32_t)(i & 1) * 128, alo + k, hi, blo + k, hi, i128); break;
        case kQk4: ptx::mma_ss_lh<true>(tmem + (uint32_t)(i & 3) * 128, alo + k, hi, blo + k, hi, i128); break;
        case kPv2: ptx::mma_ts_lh<true>(tmem + 384 + (uint32_t)(i & 1) * 64, pa, vb, hv, ipv); break;
        case kQkIss2:
        case kQkIss4: ptx::mma_ss_lh<true>(own_ss, alo + k, hi, blo + k, hi, i128); break;
        case kPvIss2:
        case kPvIss4: ptx::mma_ts_lh<true>(own_ts, pa, vb, hv, ipv); break;
        default:
          // two issuers, each with its own QK^T accumulator ([0,128) or [128,256))
          // and its own P.V accumulator ([384,448) or [448,512))
          if ((i / 2) % 3 == 0)
            ptx::mma_ss_lh<true>(own_ss, alo + k, hi, blo + k, hi, i128);
          else
            ptx::mma_ts_lh<true>(tmem + 384 + (uint32_t)warp * 64, pa, vb, hv, ipv);
          break;
      }
    }
    const long long t1 = clock64();
    ptx::tc_commit(ptx::smem_u32(&sm.bar));
    if (warp == 0) {
      const uint64_t g0 = ptx::globaltimer();
      bool done = false;
      while (!(done = ptx::mbar_try_wait(ptx::smem_u32(&sm.bar), 0)) &&
             ptx::globaltimer() - g0 < 1000000000ull) {
      }
      const long long t2 = clock64();
      out[blockIdx.x * 3 + 0] = (unsigned long long)(t1 - t0);
      out[blockIdx.x * 3 + 1] = (unsigned long long)(t2 - t0);
      out[blockIdx.x * 3 + 2] = done ? 1 : 0;
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 512);
  }
}

}  // namespace
}  // namespace wfattn

int main() {
  using namespace wfattn;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  unsigned long long *d = nullptr;
  if (cudaMalloc(&d, sizeof(unsigned long long) * 3 * sms) != cudaSuccess) return 1;
  unsigned long long *h = new unsigned long long[3 * sms];
  const size_t smem = sizeof(ProbeSmem) + 1024;
  cudaFuncSetAttribute(mma_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  printf("tcgen05.mma kind::f16, M=128, K=16, %d back-to-back MMAs per thread, %d CTAs\n",
         kIssued, sms);
  for (int c = 0; c < kCases; ++c) {
    for (int rep = 0; rep < 2; ++rep) mma_rate_kernel<<<sms, 128, smem>>>(c, d);
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      printf("CUDA error: %s\n", cudaGetErrorString(e));
      return 1;
    }
    cudaMemcpy(h, d, sizeof(unsigned long long) * 3 * sms, cudaMemcpyDeviceToHost);
    double issue = 0, total = 0;
    int ok = 1;
    for (int b = 0; b < sms; ++b) {
      issue += (double)h[3 * b];
      total += (double)h[3 * b + 1];
      ok &= (int)h[3 * b + 2];
    }
    const double cyc = total / sms / kIssued;
    printf("%-22s %7.1f cycles/MMA (issue %7.1f)  %6.0f FLOP/cycle/SM%s\n", kNames[c], cyc,
           issue / sms / kIssued, kFlop[c] / cyc, ok ? "" : "  (wait expired)");
  }
  delete[] h;
  cudaFree(d);
  return 0;
}
