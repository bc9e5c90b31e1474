/*
 * wfattn.h -- C ABI of libwfattn, the B200 (sm_100a) attention library that
 * replaces the WarpForth attention kernel (demo/attention.forth compiled to
 * demo/attention.ptx in tetsuo-cpp/warpforth) and its launch paths.
 *
 * Conventions shared by every entry point:
 *  - All tensor pointers are DEVICE pointers owned by the caller.  The library
 *    never allocates device memory on the attention paths (wfattn_peer_alloc
 *    allocates on request); outputs are fully overwritten over their logical
 *    extent.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream,
 *    which is what the reference launches on: warpforth-runner.cpp:318-319).
 *    Every call is asynchronous with respect to the host, like the reference's
 *    cuLaunchKernel.
 *  - Errors come back as a wfattn_status_t; nothing calls exit().  The text of
 *    the last failure on the calling thread is available from
 *    wfattn_last_error().  Argument checks happen on the host before any
 *    launch.
 *  - Strides are in ELEMENTS, ordered {batch, head, seq}; the head_dim stride
 *    must be 1.  A NULL stride pointer means the contiguous [B, H, S, D] layout.
 *  - Causal masking aligns the query block with the END of the key block:
 *    query i (0-based) sees keys t <= i + (seq_k - seq_q).  With
 *    seq_q == seq_k this is exactly the reference's `t > row` mask
 *    (demo/attention.forth:31-33).  Causal calls require seq_k >= seq_q.
 *  - The library is thread-safe: the only global state is a per-device
 *    status word and a per-device cache of properties, set up under a mutex.
 */
#ifndef WFATTN_H
#define WFATTN_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WFATTN_API __attribute__((visibility("default")))
#else
#define WFATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  WFATTN_OK = 0,
  WFATTN_INVALID_ARG = 1,  /* bad pointer, size, stride, alignment or geometry */
  WFATTN_UNSUPPORTED = 2,  /* valid request outside what the kernels implement */
  WFATTN_CUDA_ERROR = 3,   /* a CUDA runtime/driver call failed */
  WFATTN_TIMEOUT = 4       /* a bounded device-side wait expired (see wfattn_device_status) */
} wfattn_status_t;

typedef enum {
  WFATTN_DTYPE_F32 = 0,  /* f32 I/O; f32 arithmetic held to <= 1e-5 abs of the f64 reference */
  WFATTN_DTYPE_BF16 = 1  /* bf16 I/O; f32 accumulation on tcgen05 tensor cores */
} wfattn_dtype_t;

typedef struct {
  unsigned int x, y, z;
} wfattn_dim3;

/* Library version as 10000*major + 100*minor + patch. */
WFATTN_API int wfattn_version(void);

/* Static text for a status code. */
WFATTN_API const char *wfattn_status_string(wfattn_status_t status);

/* Message describing the last failure on the calling thread ("" if none). */
WFATTN_API const char *wfattn_last_error(void);

/*
 * Drop-in for the reference kernel launch.
 *
 * Replaces: `attention(Q, K, V, O, SEQ_LEN, HEAD_DIM)` declared at
 * demo/attention.forth:8-16 (bare-pointer ABI: lib/Conversion/Passes.cpp:42-45),
 * as launched by tools/warpforth-runner/warpforth-runner.cpp:313-319 and by
 * demo/warpforth.py:40-49.  Q, K, V, O are contiguous row-major [seq_len,
 * head_dim] f32 arrays of ONE head; O is overwritten.  The score scale is
 * 1/sqrt(head_dim) and the mask is causal, as in the reference.
 *
 * `grid` and `block` may be NULL.  When given they must be the reference's
 * geometry (seq_len, 1, 1), otherwise WFATTN_INVALID_ARG; the library then
 * picks its own launch shape.  Unlike the reference (valid for
 * 2 <= seq_len <= 1024), any seq_len >= 1 is accepted; head_dim <= 256.
 */
WFATTN_API wfattn_status_t wfattn_attention(const float *Q, const float *K, const float *V, float *O,
                                 int64_t seq_len, int64_t head_dim, const wfattn_dim3 *grid,
                                 const wfattn_dim3 *block, void *stream);

/*
 * Batched multi-head scaled-dot-product attention over [B, H, S, D] tensors
 * (prefill: every query row of every head in one launch).
 *
 * Replaces: the per-head launch loop of demo/gpt2_generate.py:42-50 (one
 * `attention` launch per head, batch index 0 only) with one call over all
 * batches and heads, reading the strided q/k/v views directly.
 *
 * dtype WFATTN_DTYPE_F32: q, k, v, o are f32; any head_dim in [1, 256].  With
 *   head_dim 64, 16-byte aligned pointers, strides that are multiples of 4
 *   elements and no zero (broadcast) strides, it runs on the tensor cores
 *   (three tf32 MMAs per product); otherwise on the CUDA cores.  Both stay
 *   within 1e-5 absolute of the f64 reference.
 * dtype WFATTN_DTYPE_BF16: q, k, v, o are bf16; head_dim must be 64; the
 *   q/k/v base pointers must be 16-byte aligned and their batch/head/seq
 *   strides multiples of 8 elements (TMA requirements).
 * scale <= 0 selects 1/sqrt(head_dim).
 */
WFATTN_API wfattn_status_t wfattn_prefill(int dtype, int64_t batch, int64_t heads, int64_t seq_q,
                               int64_t seq_k, int64_t head_dim, const void *q,
                               const int64_t *q_strides, const void *k, const int64_t *k_strides,
                               const void *v, const int64_t *v_strides, void *o,
                               const int64_t *o_strides, float scale, int causal, void *stream);

/*
 * bf16 prefill whose output is written to several buffers at once -- no
 * counterpart in the reference, which runs on one GPU; this fuses the
 * all-gather of a head-sharded multi-GPU prefill into the kernel.
 *
 * Same arguments as wfattn_prefill with dtype WFATTN_DTYPE_BF16, except that
 * the output goes to every one of outputs[0 .. n_outputs-1] (1 <= n_outputs
 * <= 8), each a [B, H, Sq, 64] bf16 view with the strides o_strides, e.g. this
 * rank's heads inside every rank's full output buffer when the buffers are
 * mapped across GPUs (wfattn_peer_alloc / wfattn_peer_open).  q, k, v and
 * outputs[0] must be device memory of the calling GPU (WFATTN_INVALID_ARG
 * otherwise): they are read and written through TMA tensor maps.
 * outputs[1..] receive untiled bulk copies (cp.async.bulk, shared -> global,
 * no multicast) of every finished 32-row output slab, so the TMA engine moves
 * the bytes over NVLink while the kernel computes the next tile.  The copies
 * are complete when the kernel is; a caller that writes into other GPUs'
 * buffers synchronises with those GPUs afterwards.
 */
WFATTN_API wfattn_status_t wfattn_prefill_gather(int64_t batch, int64_t heads, int64_t seq_q,
                                                 int64_t seq_k, int64_t head_dim, const void *q,
                                                 const int64_t *q_strides, const void *k,
                                                 const int64_t *k_strides, const void *v,
                                                 const int64_t *v_strides, void *const *outputs,
                                                 int n_outputs, const int64_t *o_strides,
                                                 float scale, int causal, void *stream);

/*
 * bf16 prefill whose output is written through a multicast (NVLS) address --
 * the same fused all-gather as wfattn_prefill_gather, with each output byte
 * leaving the GPU once: the NVLink switch copies it into every GPU's buffer.
 * No counterpart in the reference.
 *
 * Same arguments as wfattn_prefill with dtype WFATTN_DTYPE_BF16, except that
 * o_multicast is the multicast mapping, on the calling GPU, of a [B, H, Sq,
 * 64] bf16 view (strides o_strides) that every participating GPU has bound to
 * the same multicast object at the same offset (e.g. this rank's heads inside
 * a symmetric-memory output buffer); it must be 16-byte aligned.  q, k, v must
 * be device memory of the calling GPU (WFATTN_INVALID_ARG otherwise).  Each
 * finished 32-row output slab is written with multimem.st (16 bytes a thread,
 * weak, followed by a system-scope fence at the end of each thread); the
 * stores are complete when the kernel is, and the caller synchronises with the
 * other GPUs before they read their buffers.
 */
WFATTN_API wfattn_status_t wfattn_prefill_multicast(int64_t batch, int64_t heads, int64_t seq_q,
                                                    int64_t seq_k, int64_t head_dim,
                                                    const void *q, const int64_t *q_strides,
                                                    const void *k, const int64_t *k_strides,
                                                    const void *v, const int64_t *v_strides,
                                                    void *o_multicast, const int64_t *o_strides,
                                                    float scale, int causal, void *stream);

/*
 * Decode attention: one query token per (batch, head) against a padded KV
 * cache, split over key chunks and combined (split-KV).
 *
 * Replaces: nothing in the reference, which has no KV cache
 * (demo/README.md:45, demo/gpt2_generate.py:84 use_cache=False); this is the
 * decode step the GPT-2 demo would take with a cache.
 *
 * q:        bf16 [B, H, D] with strides q_strides = {batch, head} (NULL = contiguous)
 * k_cache:  bf16 [B, H, max_kv_len, D] with k_strides = {batch, head, seq};
 *           the seq stride must be D (the rows of one head are contiguous)
 * v_cache:  bf16, same shape and rule, v_strides
 * kv_lens:  DEVICE int32 [B], 1 <= kv_lens[b] <= max_kv_len (keys past
 *           kv_lens[b] are never read)
 * o:        f32 [B, H, D] with o_strides = {batch, head} (NULL = contiguous)
 * head_dim must be 64.  scale <= 0 selects 1/sqrt(head_dim).
 * batch * heads and max_kv_len must each be at most 2^31 - 1
 * (WFATTN_INVALID_ARG otherwise; wfattn_decode_workspace_size returns 0).
 * workspace: device scratch of at least wfattn_decode_workspace_size() bytes,
 *           16-byte aligned, owned by the caller; calls that share a
 *           workspace must be ordered on one stream.
 */
WFATTN_API size_t wfattn_decode_workspace_size(int64_t batch, int64_t heads, int64_t max_kv_len,
                                    int64_t head_dim);

WFATTN_API wfattn_status_t wfattn_decode(int64_t batch, int64_t heads, int64_t head_dim, int64_t max_kv_len,
                              const void *q, const int64_t *q_strides, const void *k_cache,
                              const int64_t *k_strides, const void *v_cache,
                              const int64_t *v_strides, const int32_t *kv_lens, float *o,
                              const int64_t *o_strides, float scale, void *workspace,
                              size_t workspace_bytes, void *stream);

/*
 * Decode over an f32 KV cache: the same split-KV decode as wfattn_decode with
 * f32 q, k_cache and v_cache (f32 arithmetic throughout, the f32 path's
 * accuracy contract: <= 1e-5 absolute of the f64 reference).
 *
 * Replaces: nothing in the reference (no KV cache, demo/README.md:45); this is
 * the decode step of the f32 GPT-2 demo run with use_cache=True, the cache
 * being the f32 [B, H, L, D] keys and values the model keeps.
 *
 * Arguments as wfattn_decode, with these differences: q, k_cache, v_cache are
 * f32; their strides must be multiples of 4 elements; the workspace needs
 * wfattn_decode_f32_workspace_size() bytes (keys are split into 128-key
 * chunks instead of 256).
 */
WFATTN_API size_t wfattn_decode_f32_workspace_size(int64_t batch, int64_t heads,
                                                   int64_t max_kv_len, int64_t head_dim);

WFATTN_API wfattn_status_t wfattn_decode_f32(int64_t batch, int64_t heads, int64_t head_dim,
                                             int64_t max_kv_len, const float *q,
                                             const int64_t *q_strides, const float *k_cache,
                                             const int64_t *k_strides, const float *v_cache,
                                             const int64_t *v_strides, const int32_t *kv_lens,
                                             float *o, const int64_t *o_strides, float scale,
                                             void *workspace, size_t workspace_bytes,
                                             void *stream);

/*
 * Decode without any device allocation -- no counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc: code that only holds the buffers it
 * was handed (a plugin whose host framework owns all device memory through
 * its own pool, or a foreign-language caller with no CUDA allocator of its
 * own), and decode loops that cannot afford the device synchronisation an
 * allocation may cause.  Same arguments and results as wfattn_decode, minus
 * the workspace: the split-KV partials live in a static device array of
 * 8 MiB (8,388,608 bytes) inside the library, which every GPU that loads the
 * library holds until the process exits.  Shapes needing more scratch than
 * that -- batch * heads * ceil(max_kv_len / 256) above 31,775 -- are rejected
 * with WFATTN_INVALID_ARG before any CUDA call.
 *
 * The first call on a device looks up the array's device address (with that
 * device current); make that first call before any stream capture.  All calls
 * share the one array: calls that overlap on the GPU (e.g. on two streams)
 * race and must be serialised by the caller.  Nothing in the array needs to
 * start at zero; each call writes every partial it reads.
 */
WFATTN_API wfattn_status_t wfattn_decode_noalloc(int64_t batch, int64_t heads, int64_t head_dim,
                                                 int64_t max_kv_len, const void *q,
                                                 const int64_t *q_strides, const void *k_cache,
                                                 const int64_t *k_strides, const void *v_cache,
                                                 const int64_t *v_strides,
                                                 const int32_t *kv_lens, float *o,
                                                 const int64_t *o_strides, float scale,
                                                 void *stream);

/*
 * Peer buffers -- no counterpart in the reference, which runs on one GPU.
 *
 * Device memory that other processes on the node can map, for the outputs of
 * a head-sharded prefill (wfattn_prefill_gather): every rank allocates its
 * full output buffer with wfattn_peer_alloc, sends the 64-byte handle to the
 * other ranks (any host channel), and maps theirs with wfattn_peer_open; the
 * kernel then stores straight into the mapped buffers over NVLink.  Plain
 * CUDA IPC: cudaMalloc'd memory, ordinary peer mappings, no multicast.
 *
 * wfattn_peer_alloc:  `bytes` of device memory on `device` and its handle.
 * wfattn_peer_open:   maps another process's buffer on `device` (never one's
 *                     own handle).
 * wfattn_peer_close:  unmaps a buffer returned by wfattn_peer_open.
 * wfattn_peer_free:   frees a buffer from wfattn_peer_alloc; every process
 *                     that mapped it closes its mapping first.
 * These calls synchronise as cudaMalloc / cudaFree do; the current device is
 * left as it was.
 */
typedef struct wfattn_peer_handle {
  unsigned char bytes[64];
} wfattn_peer_handle_t;

WFATTN_API wfattn_status_t wfattn_peer_alloc(size_t bytes, int device, void **ptr,
                                             wfattn_peer_handle_t *handle);
WFATTN_API wfattn_status_t wfattn_peer_open(const wfattn_peer_handle_t *handle, int device,
                                            void **ptr);
WFATTN_API wfattn_status_t wfattn_peer_close(void *ptr, int device);
WFATTN_API wfattn_status_t wfattn_peer_free(void *ptr, int device);

/*
 * Reads (and optionally clears) the device-side status word of the current
 * device: WFATTN_OK, or WFATTN_TIMEOUT when a bounded wait inside a kernel
 * (TMA/MMA pipeline barrier) gave up and the kernel returned early.
 * Synchronizes `stream` first.
 */
WFATTN_API wfattn_status_t wfattn_device_status(void *stream, int clear);

#ifdef __cplusplus
}
#endif

#endif /* WFATTN_H */
