"""Python binding of libwfattn for PyTorch tensors.

``AttentionKernel`` keeps the interface of the reference's PyCUDA wrapper
(demo/warpforth.py:16-49 in tetsuo-cpp/warpforth): construct it, then call it
with contiguous f32 CUDA tensors ``q, k, v, o`` of shape (seq_len, head_dim)
plus ``seq_len`` and ``head_dim``; ``o`` is overwritten with the causal
attention of that one head.  Instead of loading ``attention.ptx`` it calls
``wfattn_attention`` from libwfattn on torch's current stream.

``attention`` and ``decode`` are the batched forms (all batches and heads in
one launch, strided views accepted, f32 or bf16).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

from . import _lib


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


# The current stream's raw handle without building a torch.cuda.Stream object per call (the
# accessor torch's own compiled kernels use); the public call where it is absent.
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_handle(device: torch.device) -> int:
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None
                           else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")


class AttentionKernel:
    """Launches the causal attention kernel for one head (drop-in for demo/warpforth.py).

    The kernel computes ``O = softmax(Q @ K^T / sqrt(head_dim)) @ V`` with a
    causal mask, reading and writing f32.  ``ptx_path`` is accepted for
    signature compatibility with the reference wrapper and is not read: the
    kernel comes from libwfattn.
    """

    def __init__(self, ptx_path: str | Path | None = None) -> None:
        self._lib = _lib.load()
        self.ptx_path = ptx_path

    def __call__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor,
                 seq_len: int, head_dim: int) -> None:
        for name, t in (("q", q), ("k", k), ("v", v), ("o", o)):
            _require_cuda(name, t)
            if t.dtype != torch.float32:
                raise ValueError(f"{name} must be float32, got {t.dtype}")
            if not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous")
            if t.numel() < seq_len * head_dim:
                raise ValueError(f"{name} holds {t.numel()} elements, fewer than "
                                 f"seq_len*head_dim = {seq_len * head_dim}")
        geom = _lib.Dim3(int(seq_len), 1, 1)
        _lib.check(self._lib.wfattn_attention(
            _ptr(q), _ptr(k), _ptr(v), _ptr(o), int(seq_len), int(head_dim),
            ctypes.byref(geom), ctypes.byref(geom), _stream_handle(q.device)))


_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True,
              scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Batched scaled-dot-product attention over [B, H, S, D] CUDA tensors.

    q is [B, H, Sq, D], k and v are [B, H, Sk, D]; any batch/head/seq strides
    are accepted (the head_dim stride must be 1).  f32 tensors run the
    reference-accurate path (head_dim <= 256; within 1e-5 of f64): the 3xTF32
    tensor-core kernel for head_dim 64 with 16-byte aligned rows, the CUDA-core
    kernel otherwise; bf16 tensors run the tcgen05 tensor-core kernel (head_dim 64).  Causal masking aligns the
    queries with the end of the keys.  Returns ``out`` (allocated as a
    contiguous [B, H, Sq, D] tensor of q's dtype when not given).
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(name, t)
        if t.dim() != 4:
            raise ValueError(f"{name} must be [B, H, S, D], got shape {tuple(t.shape)}")
        if t.stride(3) != 1:
            raise ValueError(f"{name} must have a unit head_dim stride")
    if q.dtype not in _DTYPES or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(f"q/k/v must all be float32 or all bfloat16 (got {q.dtype}, {k.dtype}, "
                         f"{v.dtype})")
    b, h, sq, d = q.shape
    sk = k.shape[2]
    if k.shape != (b, h, sk, d) or v.shape != (b, h, sk, d):
        raise ValueError(f"shape mismatch: q {tuple(q.shape)}, k {tuple(k.shape)}, "
                         f"v {tuple(v.shape)}")
    if out is None:
        out = torch.empty((b, h, sq, d), dtype=q.dtype, device=q.device)
    elif out.shape != q.shape or out.dtype != q.dtype or out.stride(3) != 1:
        raise ValueError("out must match q's shape and dtype with a unit head_dim stride")
    lib = _lib.load()
    st = [_lib.strides_arg(t.stride()[:3]) for t in (q, k, v, out)]
    _lib.check(lib.wfattn_prefill(
        _DTYPES[q.dtype], b, h, sq, sk, d, _ptr(q), st[0], _ptr(k), st[1], _ptr(v), st[2],
        _ptr(out), st[3], float(scale) if scale else 0.0, 1 if causal else 0,
        _stream_handle(q.device)))
    return out


def _check_bf16_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(name, t)
        if t.dtype != torch.bfloat16 or t.dim() != 4 or t.stride(3) != 1:
            raise ValueError(f"{name} must be a bf16 [B, H, S, D] view with a unit last stride")
    b, h, _, d = q.shape
    sk = k.shape[2]
    if k.shape != (b, h, sk, d) or v.shape != (b, h, sk, d):
        raise ValueError("shape mismatch")


def attention_gather(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                     outs: list[torch.Tensor], *, causal: bool = True,
                     scale: float | None = None) -> None:
    """bf16 attention of q/k/v ([B, H, S, 64] CUDA views) written to every tensor in ``outs``.

    Each ``outs[i]`` is a [B, H, Sq, 64] bf16 view with the same strides.  The kernel
    stores every finished output tile to all of them.
    """
    _check_bf16_qkv(q, k, v)
    if not 1 <= len(outs) <= 8:
        raise ValueError("outs must hold 1 to 8 tensors")
    for o in outs:
        if o.shape != q.shape or o.dtype != q.dtype or o.stride() != outs[0].stride():
            raise ValueError("every output must match q's shape and dtype with one set of strides")
    attention_gather_ptrs(q, k, v, [o.data_ptr() for o in outs], outs[0].stride()[:3],
                          causal=causal, scale=scale)


def attention_gather_ptrs(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          out_ptrs: list[int], out_strides: tuple[int, int, int], *,
                          causal: bool = True, scale: float | None = None) -> None:
    """``attention_gather`` with raw output addresses: each ``out_ptrs[i]`` is the start of
    a [B, H, Sq, 64] bf16 view with element strides ``out_strides`` = (batch, head, seq),
    e.g. this rank's heads inside every rank's ``peer.PeerBuffer`` as mapped on this GPU.
    ``out_ptrs[0]`` must be this GPU's own memory, as must q, k and v (TMA tensor loads
    and stores); the others get bulk copies of each finished output slab.  The copies
    into other GPUs' buffers are complete when the kernel is; the caller synchronises
    with those GPUs afterwards."""
    _check_bf16_qkv(q, k, v)
    if not 1 <= len(out_ptrs) <= 8:
        raise ValueError("out_ptrs must hold 1 to 8 addresses")
    b, h, sq, d = q.shape
    lib = _lib.load()
    st = [_lib.strides_arg(t.stride()[:3]) for t in (q, k, v)]
    ptrs = (ctypes.c_void_p * len(out_ptrs))(*out_ptrs)
    _lib.check(lib.wfattn_prefill_gather(
        b, h, sq, k.shape[2], d, _ptr(q), st[0], _ptr(k), st[1], _ptr(v), st[2], ptrs,
        len(out_ptrs), _lib.strides_arg(out_strides), float(scale) if scale else 0.0,
        1 if causal else 0, _stream_handle(q.device)))


def attention_multicast_ptr(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out_mc: int,
                            out_strides: tuple[int, int, int], *, causal: bool = True,
                            scale: float | None = None) -> None:
    """bf16 prefill whose output goes out through a multicast (NVLS) address: ``out_mc`` is
    the start, in this GPU's multicast mapping, of a [B, H, Sq, 64] bf16 view with element
    strides ``out_strides`` = (batch, head, seq) that every rank has bound at the same
    offset (this rank's heads inside a symmetric-memory buffer).  Each output row leaves
    the GPU once and lands in every rank's buffer; q, k and v must be this GPU's memory.
    The stores are complete when the kernel is; the caller synchronises with the other
    ranks afterwards."""
    _check_bf16_qkv(q, k, v)
    b, h, sq, d = q.shape
    lib = _lib.load()
    st = [_lib.strides_arg(t.stride()[:3]) for t in (q, k, v)]
    _lib.check(lib.wfattn_prefill_multicast(
        b, h, sq, k.shape[2], d, _ptr(q), st[0], _ptr(k), st[1], _ptr(v), st[2],
        ctypes.c_void_p(out_mc), _lib.strides_arg(out_strides), float(scale) if scale else 0.0,
        1 if causal else 0, _stream_handle(q.device)))


class DecodeWorkspace:
    """Caller-owned scratch for ``decode`` (grown on demand, reused across calls)."""

    def __init__(self) -> None:
        self.buffer: torch.Tensor | None = None

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        if self.buffer is None or self.buffer.numel() < nbytes or self.buffer.device != device:
            self.buffer = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device)
        return self.buffer


def decode_workspace_size(batch: int, heads: int, max_kv_len: int, head_dim: int,
                          dtype: torch.dtype = torch.bfloat16) -> int:
    lib = _lib.load()
    fn = lib.wfattn_decode_f32_workspace_size if dtype == torch.float32 else \
        lib.wfattn_decode_workspace_size
    return int(fn(batch, heads, max_kv_len, head_dim))


def decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, kv_lens: torch.Tensor,
           *, scale: float | None = None, out: torch.Tensor | None = None,
           workspace: DecodeWorkspace | None = None) -> torch.Tensor:
    """One-token decode attention over a padded KV cache (split-KV).

    q: [B, H, D] or [B, H, 1, D]; k_cache / v_cache: [B, H, Lmax, D] with
    contiguous rows; all three bf16 (``wfattn_decode``) or all f32
    (``wfattn_decode_f32``, the reference-accurate path); kv_lens: int32 CUDA
    [B] with 1 <= kv_lens[b] <= Lmax.  Returns f32 [B, H, D].
    """
    if q.dim() == 4:
        q = q[:, :, 0, :]
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache), ("kv_lens", kv_lens)):
        _require_cuda(name, t)
    if q.dtype not in (torch.bfloat16, torch.float32) or k_cache.dtype != q.dtype or \
            v_cache.dtype != q.dtype:
        raise ValueError("decode expects q / k_cache / v_cache all bfloat16 or all float32")
    if kv_lens.dtype != torch.int32:
        raise ValueError("kv_lens must be int32")
    b, h, d = q.shape
    lmax = k_cache.shape[2]
    if k_cache.shape != (b, h, lmax, d) or v_cache.shape != (b, h, lmax, d):
        raise ValueError("cache shape mismatch")
    if out is None:
        out = torch.empty((b, h, d), dtype=torch.float32, device=q.device)
    ws = (workspace or DecodeWorkspace()).get(decode_workspace_size(b, h, lmax, d, q.dtype),
                                              q.device)
    lib = _lib.load()
    qs = _lib.strides_arg(q.stride()[:2])
    ks = _lib.strides_arg(k_cache.stride()[:3])
    vs = _lib.strides_arg(v_cache.stride()[:3])
    os_ = _lib.strides_arg(out.stride()[:2])
    fn = lib.wfattn_decode_f32 if q.dtype == torch.float32 else lib.wfattn_decode
    _lib.check(fn(
        b, h, d, lmax, _ptr(q), qs, _ptr(k_cache), ks, _ptr(v_cache), vs, _ptr(kv_lens),
        _ptr(out), os_, float(scale) if scale else 0.0, _ptr(ws), ws.numel(),
        _stream_handle(q.device)))
    return out


def device_status(clear: bool = True) -> None:
    """Raise if a kernel on the current device recorded a device-side failure."""
    lib = _lib.load()
    _lib.check(lib.wfattn_device_status(_stream_handle(torch.device("cuda")), 1 if clear else 0))
