// wfattn_api.cu -- the C ABI of libwfattn (include/wfattn.h): argument
// validation, per-device setup, dispatch to the kernels, error reporting.
//
// Error behaviour follows the reference's contract where it has one (the
// caller owns every buffer, launches are asynchronous, the kernel allocates
// nothing) and replaces its `exit(1)` on failure
// (tools/warpforth-runner/warpforth-runner.cpp:28-38) with status codes.
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>
#include <vector>

#include "../../include/wfattn.h"
#include "wfattn_internal.h"

namespace wfattn {

// One status word per device.  Kernels OR bits into it when a bounded wait
// expires; wfattn_device_status() reads and clears it.
__device__ unsigned int g_device_status;

namespace {

thread_local std::string t_last_error;

std::mutex g_dev_mutex;
std::vector<DeviceInfo> g_devices;  // indexed by device ordinal; sm_count == 0 means unset

wfattn_status_t fail(wfattn_status_t st, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return st;
}

wfattn_status_t cuda_fail(cudaError_t err, const char *what) {
  return fail(WFATTN_CUDA_ERROR, "%s: %s (%s)", what, cudaGetErrorName(err),
              cudaGetErrorString(err));
}

// Looks up (and on first use sets up) the properties of the current device.
wfattn_status_t current_device(DeviceInfo *out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if ((int)g_devices.size() <= dev) g_devices.resize(dev + 1, DeviceInfo{});
  DeviceInfo &d = g_devices[dev];
  if (d.sm_count == 0) {
    cudaDeviceProp prop;
    err = cudaGetDeviceProperties(&prop, dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetDeviceProperties");
    void *status = nullptr;
    err = cudaGetSymbolAddress(&status, g_device_status);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(status)");
    d.device = dev;
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    d.smem_optin = prop.sharedMemPerBlockOptin;
    d.status = static_cast<unsigned int *>(status);
    d.sm_count = prop.multiProcessorCount;
  }
  *out = d;
  return WFATTN_OK;
}

bool is_sm100(const DeviceInfo &d) { return d.cc_major == 10 && d.cc_minor == 0; }

Strides3 resolve_strides(const int64_t *s, int64_t H, int64_t S, int64_t D) {
  if (s) return Strides3{s[0], s[1], s[2]};
  return Strides3{H * S * D, S * D, D};
}

bool strides_ok(const Strides3 &s) { return s.b >= 0 && s.h >= 0 && s.s >= 0; }

float resolve_scale(float scale, int64_t D) {
  return scale > 0.f ? scale : (float)(1.0 / sqrt((double)D));
}

// Layout rules of the bf16 tensor-core kernels (TMA tensor maps).
wfattn_status_t check_bf16(const PrefillArgs &a) {
  if (a.D != 64) return fail(WFATTN_UNSUPPORTED, "bf16 path supports head_dim == 64 only");
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(a.q) || !al16(a.k) || !al16(a.v) || (a.o && !al16(a.o)))
    return fail(WFATTN_INVALID_ARG, "bf16 tensors must be 16-byte aligned");
  for (int r = 0; r < a.n_peers; ++r)
    if (!a.o_peers[r] || !al16(a.o_peers[r]))
      return fail(WFATTN_INVALID_ARG, "output %d is null or not 16-byte aligned", r);
  const Strides3 *all[4] = {&a.qs, &a.ks, &a.vs, &a.os};
  for (const Strides3 *x : all)
    if (x->b % 8 || x->h % 8 || x->s % 8)
      return fail(WFATTN_INVALID_ARG, "bf16 strides must be multiples of 8 elements");
  const int64_t ext_q[3] = {a.B, a.H, a.Sq}, ext_k[3] = {a.B, a.H, a.Sk};
  for (int i = 0; i < 3; ++i) {
    const int64_t sq[3] = {a.qs.b, a.qs.h, a.qs.s}, sk[3] = {a.ks.b, a.ks.h, a.ks.s},
                  sv[3] = {a.vs.b, a.vs.h, a.vs.s}, so[3] = {a.os.b, a.os.h, a.os.s};
    if ((ext_q[i] > 1 && (sq[i] == 0 || so[i] == 0)) ||
        (ext_k[i] > 1 && (sk[i] == 0 || sv[i] == 0)))
      return fail(WFATTN_INVALID_ARG, "bf16 path does not take zero (broadcast) strides");
  }
  return WFATTN_OK;
}

}  // namespace

namespace {
struct SmemAttr {
  const void *func;
  int device, bytes;
};
std::mutex g_attr_mutex;
std::vector<SmemAttr> g_attrs;
}  // namespace

cudaError_t ensure_smem_attr(const void *func, int bytes, int device) {
  std::lock_guard<std::mutex> lock(g_attr_mutex);
  for (const SmemAttr &a : g_attrs)
    if (a.func == func && a.device == device && a.bytes == bytes) return cudaSuccess;
  const cudaError_t err =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess) g_attrs.push_back(SmemAttr{func, device, bytes});
  return err;
}

#ifdef WFATTN_TRACE
cudaError_t set_trace_prefill_1q(void *p);
cudaError_t set_trace_prefill_2q(void *p);
#endif
}  // namespace wfattn

using namespace wfattn;

extern "C" {

int wfattn_version(void) { return 100; }

const char *wfattn_status_string(wfattn_status_t status) {
  switch (status) {
    case WFATTN_OK: return "ok";
    case WFATTN_INVALID_ARG: return "invalid argument";
    case WFATTN_UNSUPPORTED: return "unsupported";
    case WFATTN_CUDA_ERROR: return "cuda error";
    case WFATTN_TIMEOUT: return "device wait timed out";
  }
  return "unknown status";
}

const char *wfattn_last_error(void) { return t_last_error.c_str(); }

}  // extern "C"

namespace {

// Argument checks and setup shared by the prefill entry points.
wfattn_status_t prepare_prefill(int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k,
                                int64_t head_dim, const void *q, const int64_t *q_strides,
                                const void *k, const int64_t *k_strides, const void *v,
                                const int64_t *v_strides, void *o, const int64_t *o_strides,
                                float scale, int causal, PrefillArgs *a, DeviceInfo *dev) {
  if (!q || !k || !v) return fail(WFATTN_INVALID_ARG, "null tensor pointer");
  if (batch < 1 || heads < 1 || seq_q < 1 || seq_k < 1 || head_dim < 1)
    return fail(WFATTN_INVALID_ARG, "sizes must be >= 1 (B=%lld H=%lld Sq=%lld Sk=%lld D=%lld)",
                (long long)batch, (long long)heads, (long long)seq_q, (long long)seq_k,
                (long long)head_dim);
  if (causal && seq_k < seq_q)
    return fail(WFATTN_INVALID_ARG, "causal attention needs seq_k >= seq_q (%lld < %lld)",
                (long long)seq_k, (long long)seq_q);
  if (!(scale == scale)) return fail(WFATTN_INVALID_ARG, "scale is NaN");
  a->B = batch;
  a->H = heads;
  a->Sq = seq_q;
  a->Sk = seq_k;
  a->D = head_dim;
  a->q = q;
  a->k = k;
  a->v = v;
  a->o = o;
  a->qs = resolve_strides(q_strides, heads, seq_q, head_dim);
  a->ks = resolve_strides(k_strides, heads, seq_k, head_dim);
  a->vs = resolve_strides(v_strides, heads, seq_k, head_dim);
  a->os = resolve_strides(o_strides, heads, seq_q, head_dim);
  if (!strides_ok(a->qs) || !strides_ok(a->ks) || !strides_ok(a->vs) || !strides_ok(a->os))
    return fail(WFATTN_INVALID_ARG, "negative stride");
  a->scale = resolve_scale(scale, head_dim);
  a->causal = causal ? 1 : 0;
  wfattn_status_t st = current_device(dev);
  if (st != WFATTN_OK) return st;
  if (!is_sm100(*dev))
    return fail(WFATTN_UNSUPPORTED, "libwfattn is built for sm_100a; device %d is sm_%d%d",
                dev->device, dev->cc_major, dev->cc_minor);
  return WFATTN_OK;
}

}  // namespace

extern "C" {

wfattn_status_t wfattn_prefill(int dtype, int64_t batch, int64_t heads, int64_t seq_q,
                               int64_t seq_k, int64_t head_dim, const void *q,
                               const int64_t *q_strides, const void *k, const int64_t *k_strides,
                               const void *v, const int64_t *v_strides, void *o,
                               const int64_t *o_strides, float scale, int causal, void *stream) {
  t_last_error.clear();
  if (!o) return fail(WFATTN_INVALID_ARG, "null tensor pointer");
  PrefillArgs a;
  DeviceInfo dev;
  wfattn_status_t st = prepare_prefill(batch, heads, seq_q, seq_k, head_dim, q, q_strides, k,
                                       k_strides, v, v_strides, o, o_strides, scale, causal, &a,
                                       &dev);
  if (st != WFATTN_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  if (dtype == WFATTN_DTYPE_F32) {
    if (head_dim > 256) return fail(WFATTN_UNSUPPORTED, "f32 path supports head_dim <= 256");
    // head_dim 64 with 16-byte aligned rows: the tensor-core kernel (3xTF32);
    // anything else: the CUDA-core kernel.  Both hold the 1e-5 contract.
    err = prefill_f32_tc_supported(a) ? launch_prefill_f32_tc(a, dev, s)
                                      : launch_prefill_f32(a, dev, s);
    if (err != cudaSuccess) return cuda_fail(err, "prefill_f32 launch");
    return WFATTN_OK;
  }
  if (dtype == WFATTN_DTYPE_BF16) {
    st = check_bf16(a);
    if (st != WFATTN_OK) return st;
    // Two 128-row query tiles per CTA (one CTA per SM) halve the K/V traffic
    // per FLOP; when that grid would not even give every SM a CTA, one tile
    // per CTA (two CTAs per SM) spreads the few rows over twice the SMs and
    // halves the longest CTA.
    const int64_t two_tile_ctas = (a.Sq + 255) / 256 * a.B * a.H;
    err = two_tile_ctas < dev.sm_count ? launch_prefill_bf16_1q(a, dev, s)
                                       : launch_prefill_bf16_2q(a, dev, s);
    if (err != cudaSuccess) return cuda_fail(err, "prefill_bf16 launch");
    return WFATTN_OK;
  }
  return fail(WFATTN_INVALID_ARG, "unknown dtype %d", dtype);
}

wfattn_status_t wfattn_prefill_gather(int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_k,
                                      int64_t head_dim, const void *q, const int64_t *q_strides,
                                      const void *k, const int64_t *k_strides, const void *v,
                                      const int64_t *v_strides, void *const *outputs,
                                      int n_outputs, const int64_t *o_strides, float scale,
                                      int causal, void *stream) {
  t_last_error.clear();
  if (!outputs || n_outputs < 1 || n_outputs > kMaxOutputPeers)
    return fail(WFATTN_INVALID_ARG, "n_outputs must be in [1, %d] with an output array",
                kMaxOutputPeers);
  PrefillArgs a;
  DeviceInfo dev;
  wfattn_status_t st = prepare_prefill(batch, heads, seq_q, seq_k, head_dim, q, q_strides, k,
                                       k_strides, v, v_strides, nullptr, o_strides, scale,
                                       causal, &a, &dev);
  if (st != WFATTN_OK) return st;
  a.o_peers = outputs;
  a.n_peers = n_outputs;
  st = check_bf16(a);
  if (st != WFATTN_OK) return st;
  // q, k, v (TMA loads) and outputs[0] (TMA tensor stores) must be this GPU's
  // own memory: the kernel reaches other GPUs' buffers only through the
  // untiled bulk copies to outputs[1..].
  const void *local[4] = {q, k, v, outputs[0]};
  const char *names[4] = {"q", "k", "v", "outputs[0]"};
  for (int i = 0; i < 4; ++i) {
    cudaPointerAttributes attr;
    const cudaError_t perr = cudaPointerGetAttributes(&attr, local[i]);
    if (perr != cudaSuccess) {
      cudaGetLastError();
      return cuda_fail(perr, "cudaPointerGetAttributes");
    }
    if (attr.type != cudaMemoryTypeDevice || attr.device != dev.device)
      return fail(WFATTN_INVALID_ARG, "%s must be device memory of the calling GPU (%d)",
                  names[i], dev.device);
  }
  cudaError_t err = launch_prefill_bf16_2q(a, dev, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "prefill_bf16 launch");
  return WFATTN_OK;
}

wfattn_status_t wfattn_prefill_multicast(int64_t batch, int64_t heads, int64_t seq_q,
                                         int64_t seq_k, int64_t head_dim, const void *q,
                                         const int64_t *q_strides, const void *k,
                                         const int64_t *k_strides, const void *v,
                                         const int64_t *v_strides, void *o_multicast,
                                         const int64_t *o_strides, float scale, int causal,
                                         void *stream) {
  t_last_error.clear();
  if (!o_multicast || (reinterpret_cast<uintptr_t>(o_multicast) & 15u))
    return fail(WFATTN_INVALID_ARG, "o_multicast must be a non-null, 16-byte aligned address");
  PrefillArgs a;
  DeviceInfo dev;
  wfattn_status_t st = prepare_prefill(batch, heads, seq_q, seq_k, head_dim, q, q_strides, k,
                                       k_strides, v, v_strides, nullptr, o_strides, scale,
                                       causal, &a, &dev);
  if (st != WFATTN_OK) return st;
  a.o_mc = o_multicast;
  st = check_bf16(a);
  if (st != WFATTN_OK) return st;
  // q, k, v are read through TMA tensor maps: this GPU's own memory only.
  const void *local[3] = {q, k, v};
  const char *names[3] = {"q", "k", "v"};
  for (int i = 0; i < 3; ++i) {
    cudaPointerAttributes attr;
    const cudaError_t perr = cudaPointerGetAttributes(&attr, local[i]);
    if (perr != cudaSuccess) {
      cudaGetLastError();
      return cuda_fail(perr, "cudaPointerGetAttributes");
    }
    if (attr.type != cudaMemoryTypeDevice || attr.device != dev.device)
      return fail(WFATTN_INVALID_ARG, "%s must be device memory of the calling GPU (%d)",
                  names[i], dev.device);
  }
  cudaError_t err = launch_prefill_bf16_2q(a, dev, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "prefill_bf16 launch");
  return WFATTN_OK;
}

wfattn_status_t wfattn_attention(const float *Q, const float *K, const float *V, float *O,
                                 int64_t seq_len, int64_t head_dim, const wfattn_dim3 *grid,
                                 const wfattn_dim3 *block, void *stream) {
  t_last_error.clear();
  if (seq_len < 1 || head_dim < 1)
    return fail(WFATTN_INVALID_ARG, "SEQ_LEN and HEAD_DIM must be >= 1 (got %lld, %lld)",
                (long long)seq_len, (long long)head_dim);
  auto is_ref_geom = [seq_len](const wfattn_dim3 *g) {
    return g->x == (unsigned long long)seq_len && g->y == 1 && g->z == 1;
  };
  if (grid && !is_ref_geom(grid))
    return fail(WFATTN_INVALID_ARG, "grid (%u,%u,%u) is not the kernel's (SEQ_LEN,1,1)", grid->x,
                grid->y, grid->z);
  if (block && !is_ref_geom(block))
    return fail(WFATTN_INVALID_ARG, "block (%u,%u,%u) is not the kernel's (SEQ_LEN,1,1)",
                block->x, block->y, block->z);
  return wfattn_prefill(WFATTN_DTYPE_F32, 1, 1, seq_len, seq_len, head_dim, Q, nullptr, K,
                        nullptr, V, nullptr, O, nullptr, 0.f, 1, stream);
}

size_t wfattn_decode_workspace_size(int64_t batch, int64_t heads, int64_t max_kv_len,
                                    int64_t head_dim) {
  if (head_dim < 1) return 0;
  return decode_workspace_bytes(batch, heads, max_kv_len, head_dim, false);  // 0: bad shape
}

size_t wfattn_decode_f32_workspace_size(int64_t batch, int64_t heads, int64_t max_kv_len,
                                        int64_t head_dim) {
  if (head_dim < 1) return 0;
  return decode_workspace_bytes(batch, heads, max_kv_len, head_dim, true);  // 0: bad shape
}

}  // extern "C"

namespace {

// Argument checks and launch shared by the bf16 and f32 decode entry points.
wfattn_status_t decode_common(bool f32, int64_t batch, int64_t heads, int64_t head_dim,
                              int64_t max_kv_len, const void *q, const int64_t *q_strides,
                              const void *k_cache, const int64_t *k_strides, const void *v_cache,
                              const int64_t *v_strides, const int32_t *kv_lens, float *o,
                              const int64_t *o_strides, float scale, void *workspace,
                              size_t workspace_bytes, void *stream) {
  if (!q || !k_cache || !v_cache || !kv_lens || !o)
    return fail(WFATTN_INVALID_ARG, "null tensor pointer");
  if (batch < 1 || heads < 1 || max_kv_len < 1 || head_dim < 1)
    return fail(WFATTN_INVALID_ARG, "sizes must be >= 1");
  if (!decode_shape_ok(batch, heads, max_kv_len))
    return fail(WFATTN_INVALID_ARG,
                "decode needs batch*heads <= 2^31-1 and max_kv_len <= 2^31-1 (B=%lld H=%lld "
                "max_kv_len=%lld)", (long long)batch, (long long)heads, (long long)max_kv_len);
  if (head_dim != 64) return fail(WFATTN_UNSUPPORTED, "decode supports head_dim == 64 only");
  const size_t need = decode_workspace_bytes(batch, heads, max_kv_len, head_dim, f32);
  if (!workspace || workspace_bytes < need)
    return fail(WFATTN_INVALID_ARG, "workspace of %zu bytes needed, %zu given", need,
                workspace ? workspace_bytes : (size_t)0);
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(q) || !al16(k_cache) || !al16(v_cache) || !al16(o) || !al16(workspace))
    return fail(WFATTN_INVALID_ARG, "decode tensors and workspace must be 16-byte aligned");
  DecodeArgs a;
  a.f32 = f32;
  a.B = batch;
  a.H = heads;
  a.D = head_dim;
  a.max_len = max_kv_len;
  a.q = q;
  a.qs = q_strides ? Strides3{q_strides[0], q_strides[1], 0} : Strides3{heads * head_dim, head_dim, 0};
  a.k = k_cache;
  a.v = v_cache;
  a.ks = resolve_strides(k_strides, heads, max_kv_len, head_dim);
  a.vs = resolve_strides(v_strides, heads, max_kv_len, head_dim);
  a.kv_lens = kv_lens;
  a.o = o;
  a.os = o_strides ? Strides3{o_strides[0], o_strides[1], 0} : Strides3{heads * head_dim, head_dim, 0};
  a.scale = resolve_scale(scale, head_dim);
  a.workspace = workspace;
  a.workspace_bytes = workspace_bytes;
  if (!strides_ok(a.qs) || !strides_ok(a.ks) || !strides_ok(a.vs) || !strides_ok(a.os))
    return fail(WFATTN_INVALID_ARG, "negative stride");
  // 16-byte aligned rows for the bulk copies: 8 bf16 or 4 f32 elements
  const int64_t m = f32 ? 4 : 8;
  if (a.qs.b % m || a.qs.h % m || a.ks.b % m || a.ks.h % m || a.ks.s % m || a.vs.b % m ||
      a.vs.h % m || a.vs.s % m)
    return fail(WFATTN_INVALID_ARG, "%s q/k/v strides must be multiples of %d elements",
                f32 ? "f32" : "bf16", (int)m);
  if (a.ks.s != head_dim || a.vs.s != head_dim)
    return fail(WFATTN_UNSUPPORTED, "decode needs contiguous cache rows (seq stride == head_dim)");
  if (a.os.b % 4 || a.os.h % 4)
    return fail(WFATTN_INVALID_ARG, "f32 output strides must be multiples of 4 elements");
  DeviceInfo dev;
  wfattn_status_t st = current_device(&dev);
  if (st != WFATTN_OK) return st;
  if (!is_sm100(dev))
    return fail(WFATTN_UNSUPPORTED, "libwfattn is built for sm_100a; device %d is sm_%d%d",
                dev.device, dev.cc_major, dev.cc_minor);
  cudaError_t err = launch_decode(a, dev, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "decode launch");
  return WFATTN_OK;
}

}  // namespace

extern "C" {

wfattn_status_t wfattn_decode(int64_t batch, int64_t heads, int64_t head_dim, int64_t max_kv_len,
                              const void *q, const int64_t *q_strides, const void *k_cache,
                              const int64_t *k_strides, const void *v_cache,
                              const int64_t *v_strides, const int32_t *kv_lens, float *o,
                              const int64_t *o_strides, float scale, void *workspace,
                              size_t workspace_bytes, void *stream) {
  t_last_error.clear();
  return decode_common(false, batch, heads, head_dim, max_kv_len, q, q_strides, k_cache,
                       k_strides, v_cache, v_strides, kv_lens, o, o_strides, scale, workspace,
                       workspace_bytes, stream);
}

wfattn_status_t wfattn_decode_f32(int64_t batch, int64_t heads, int64_t head_dim,
                                  int64_t max_kv_len, const float *q, const int64_t *q_strides,
                                  const float *k_cache, const int64_t *k_strides,
                                  const float *v_cache, const int64_t *v_strides,
                                  const int32_t *kv_lens, float *o, const int64_t *o_strides,
                                  float scale, void *workspace, size_t workspace_bytes,
                                  void *stream) {
  t_last_error.clear();
  return decode_common(true, batch, heads, head_dim, max_kv_len, q, q_strides, k_cache,
                       k_strides, v_cache, v_strides, kv_lens, o, o_strides, scale, workspace,
                       workspace_bytes, stream);
}

// Decode for callers that cannot allocate device memory: the split-KV
// partials go to a static device array instead of a caller workspace, then
// the ordinary decode path runs on it.  Checks the size against the array
// before any CUDA call; looks the array's address up on the first call per
// device (with that device current).
wfattn_status_t wfattn_decode_noalloc(int64_t batch, int64_t heads, int64_t head_dim,
                                      int64_t max_kv_len, const void *q,
                                      const int64_t *q_strides, const void *k_cache,
                                      const int64_t *k_strides, const void *v_cache,
                                      const int64_t *v_strides, const int32_t *kv_lens, float *o,
                                      const int64_t *o_strides, float scale, void *stream) {
  t_last_error.clear();
  if (batch < 1 || heads < 1 || max_kv_len < 1 || head_dim < 1)
    return fail(WFATTN_INVALID_ARG, "sizes must be >= 1");
  if (!decode_shape_ok(batch, heads, max_kv_len))
    return fail(WFATTN_INVALID_ARG,
                "decode needs batch*heads <= 2^31-1 and max_kv_len <= 2^31-1 (B=%lld H=%lld "
                "max_kv_len=%lld)", (long long)batch, (long long)heads, (long long)max_kv_len);
  const size_t need = decode_workspace_bytes(batch, heads, max_kv_len, head_dim, false);
  if (need > kDecodeNoAllocScratchBytes)
    return fail(WFATTN_INVALID_ARG,
                "wfattn_decode_noalloc: this shape needs %zu bytes of scratch but the static "
                "scratch holds %zu (batch*heads*ceil(max_kv_len/256) must be <= %zu); use "
                "wfattn_decode with a caller workspace",
                need, kDecodeNoAllocScratchBytes,
                kDecodeNoAllocScratchBytes / (size_t)((64 + 2) * sizeof(float)));
  void *scratch = nullptr;
  const cudaError_t err = decode_noalloc_scratch(&scratch);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(decode scratch)");
  return wfattn_decode(batch, heads, head_dim, max_kv_len, q, q_strides, k_cache, k_strides,
                       v_cache, v_strides, kv_lens, o, o_strides, scale, scratch,
                       kDecodeNoAllocScratchBytes, stream);
}

#ifdef WFATTN_TRACE
// Debug builds only: route the kernels' progress trace to `host_mapped`
// (cudaHostAllocMapped memory of at least 8 words per CTA), or NULL to stop.
__attribute__((visibility("default"))) int wfattn_debug_set_trace(void *host_mapped) {
  void *dev = nullptr;
  if (host_mapped && cudaHostGetDevicePointer(&dev, host_mapped, 0) != cudaSuccess) return 1;
  if (set_trace_prefill_1q(dev) != cudaSuccess) return 2;
  if (set_trace_prefill_2q(dev) != cudaSuccess) return 3;
  return 0;
}
#endif

wfattn_status_t wfattn_device_status(void *stream, int clear) {
  t_last_error.clear();
  cudaError_t err = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "cudaStreamSynchronize");
  unsigned int word = 0;
  err = cudaMemcpyFromSymbol(&word, g_device_status, sizeof(word));
  if (err != cudaSuccess) return cuda_fail(err, "read device status");
  if (clear && word) {
    const unsigned int zero = 0;
    err = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero));
    if (err != cudaSuccess) return cuda_fail(err, "clear device status");
  }
  if (word & kDevTimeoutMask)
    return fail(WFATTN_TIMEOUT, "a kernel's bounded wait expired (status word 0x%x)", word);
  if (word & kDevBadLengthMask)
    return fail(WFATTN_INVALID_ARG, "a kv_lens entry was outside [1, max_kv_len] (status 0x%x)",
                word);
  return WFATTN_OK;
}

// Peer buffers: plain cudaMalloc memory exported and imported with CUDA IPC
// handles.  An imported buffer is an ordinary peer mapping over NVLink; no
// multicast object is involved.
static_assert(sizeof(wfattn_peer_handle_t) == sizeof(cudaIpcMemHandle_t),
              "wfattn_peer_handle_t must hold a cudaIpcMemHandle_t");

namespace {

// Makes `device` current for the lifetime of the guard, then restores the previous device.
struct DeviceScope {
  int prev = -1;
  cudaError_t enter(int device) {
    cudaError_t err = cudaGetDevice(&prev);
    if (err != cudaSuccess) {
      prev = -1;
      return err;
    }
    return cudaSetDevice(device);
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace

wfattn_status_t wfattn_peer_alloc(size_t bytes, int device, void **ptr,
                                  wfattn_peer_handle_t *handle) {
  t_last_error.clear();
  if (!ptr || !handle || bytes == 0 || device < 0)
    return fail(WFATTN_INVALID_ARG, "peer_alloc needs bytes > 0, a device and out pointers");
  *ptr = nullptr;
  DeviceScope scope;
  cudaError_t err = scope.enter(device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
  void *p = nullptr;
  err = cudaMalloc(&p, bytes);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMalloc(peer buffer)");
  cudaIpcMemHandle_t h;
  err = cudaIpcGetMemHandle(&h, p);
  if (err != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(err, "cudaIpcGetMemHandle");
  }
  memcpy(handle->bytes, &h, sizeof(h));
  *ptr = p;
  return WFATTN_OK;
}

wfattn_status_t wfattn_peer_open(const wfattn_peer_handle_t *handle, int device, void **ptr) {
  t_last_error.clear();
  if (!ptr || !handle || device < 0)
    return fail(WFATTN_INVALID_ARG, "peer_open needs a handle, a device and an out pointer");
  *ptr = nullptr;
  DeviceScope scope;
  cudaError_t err = scope.enter(device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->bytes, sizeof(h));
  err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return cuda_fail(err, "cudaIpcOpenMemHandle");
  return WFATTN_OK;
}

wfattn_status_t wfattn_peer_close(void *ptr, int device) {
  t_last_error.clear();
  if (!ptr || device < 0) return fail(WFATTN_INVALID_ARG, "peer_close needs a pointer");
  DeviceScope scope;
  cudaError_t err = scope.enter(device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
  err = cudaIpcCloseMemHandle(ptr);
  if (err != cudaSuccess) return cuda_fail(err, "cudaIpcCloseMemHandle");
  return WFATTN_OK;
}

wfattn_status_t wfattn_peer_free(void *ptr, int device) {
  t_last_error.clear();
  if (!ptr || device < 0) return fail(WFATTN_INVALID_ARG, "peer_free needs a pointer");
  DeviceScope scope;
  cudaError_t err = scope.enter(device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
  err = cudaFree(ptr);
  if (err != cudaSuccess) return cuda_fail(err, "cudaFree(peer buffer)");
  return WFATTN_OK;
}

}  // extern "C"
