"""CPU oracle for WarpForth's causal attention kernel -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm import this package, and only as the checker or as the timed CPU
baseline.  The shipped library (``warpforth_b200``) never imports it and has no
CPU fallback.

Two restatements of ``demo/attention.forth:18-81`` (reference tree
tetsuo-cpp/warpforth) live here:

* ``wf_oracle.c`` (built into ``oracle/build/libwforacle.so`` by ``make``): the
  literal per-head restatement (``attention_head``) and the batched/strided
  generalisation (``attention``), f64 arithmetic in the kernel's order.
* ``attention_np``: a vectorised NumPy f64 form of the same math, used to
  cross-check the C build and for quick small cases.

The oracle is pinned against the reference's own attention tests
(``gpu_test/test_kernels.py:651-875``) through ``tests/golden/``.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "build" / "libwforacle.so"
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)


def build() -> Path:
    """Compile wf_oracle.c with the committed Makefile, and copy the reference's compiled
    attention kernel into ``_ref/`` where the reference tree is present (``make ref``)."""
    subprocess.run(["make", "-C", str(_HERE), "all", "ref"], check=True, capture_output=True,
                   text=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        build()
    lib = ctypes.CDLL(str(_LIB_PATH))
    lib.wfo_attention_head.restype = ctypes.c_int
    lib.wfo_attention_head.argtypes = [_f32p, _f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64]
    _f64p = ctypes.POINTER(ctypes.c_double)
    lib.wfo_attention_head_f64.restype = ctypes.c_int
    lib.wfo_attention_head_f64.argtypes = [_f64p, _f64p, _f64p, _f64p, ctypes.c_int64,
                                           ctypes.c_int64]
    lib.wfo_attention.restype = ctypes.c_int
    lib.wfo_attention.argtypes = [
        _f32p, _f32p, _f32p, _f32p,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        _i64p, _i64p, _i64p, _i64p,
        ctypes.c_double, ctypes.c_int, _i32p,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
    ]
    lib.wfo_max_threads.restype = ctypes.c_int
    _lib = lib
    return lib


def max_threads() -> int:
    return int(_load().wfo_max_threads())


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(_f32p)


def attention_head(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Literal restatement of demo/attention.forth for one head ([S, D] f32 in, f32 out)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    s, d = q.shape
    if k.shape != (s, d) or v.shape != (s, d):
        raise ValueError("q, k, v must all be [S, D]")
    o = np.empty_like(q)
    rc = _load().wfo_attention_head(_fptr(q), _fptr(k), _fptr(v), _fptr(o), s, d)
    if rc != 0:
        raise RuntimeError(f"wfo_attention_head failed ({rc})")
    return o


def attention_head_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Literal restatement with f64 I/O (the reference's f64 test twin of the kernel)."""
    q, k, v = (np.ascontiguousarray(a, dtype=np.float64) for a in (q, k, v))
    s, d = q.shape
    if k.shape != (s, d) or v.shape != (s, d):
        raise ValueError("q, k, v must all be [S, D]")
    o = np.empty_like(q)
    p = ctypes.POINTER(ctypes.c_double)
    rc = _load().wfo_attention_head_f64(q.ctypes.data_as(p), k.ctypes.data_as(p),
                                        v.ctypes.data_as(p), o.ctypes.data_as(p), s, d)
    if rc != 0:
        raise RuntimeError(f"wfo_attention_head_f64 failed ({rc})")
    return o


def _estrides(a: np.ndarray) -> np.ndarray:
    return np.array([st // a.itemsize for st in a.strides[:3]], dtype=np.int64)


def attention(q, k, v, *, scale: float | None = None, causal: bool = True, kv_lens=None,
              bh_range: tuple[int, int] | None = None, row_range: tuple[int, int] | None = None,
              nthreads: int = 0, out: np.ndarray | None = None) -> np.ndarray:
    """Batched oracle on [B, H, S, D] f32 arrays (any batch/head/seq strides, unit D stride).

    ``scale=None`` follows the reference kernel (divide by sqrt(D)); causal masking
    aligns the queries with the end of the keys; ``kv_lens`` gives per-batch
    valid key counts (decode over a padded cache).  Rows outside ``row_range`` /
    heads outside ``bh_range`` are left untouched in ``out``.
    """
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    for a in (q, k, v):
        if a.ndim != 4 or a.strides[3] != 4:
            raise ValueError("expected [B, H, S, D] float32 arrays with unit D stride")
    b, h, sq, d = q.shape
    sk = k.shape[2]
    if out is None:
        out = np.zeros((b, h, sq, d), dtype=np.float32)
    lens = None
    if kv_lens is not None:
        lens = np.ascontiguousarray(kv_lens, dtype=np.int32)
    qs, ks, vs, os_ = (_estrides(a) for a in (q, k, v, out))
    bh0, bh1 = bh_range if bh_range is not None else (-1, -1)
    r0, r1 = row_range if row_range is not None else (-1, -1)
    rc = _load().wfo_attention(
        _fptr(q), _fptr(k), _fptr(v), _fptr(out), b, h, sq, sk, d,
        qs.ctypes.data_as(_i64p), ks.ctypes.data_as(_i64p), vs.ctypes.data_as(_i64p),
        os_.ctypes.data_as(_i64p), float(scale) if scale else 0.0, int(causal),
        lens.ctypes.data_as(_i32p) if lens is not None else None,
        bh0, bh1, r0, r1, int(nthreads))
    if rc != 0:
        raise RuntimeError(f"wfo_attention failed ({rc})")
    return out


def attention_np(q, k, v, *, scale: float | None = None, causal: bool = True,
                 kv_lens=None) -> np.ndarray:
    """Vectorised f64 NumPy form of the same computation ([B, H, S, D] in, f32 out)."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    b, h, sq, d = q.shape
    sk = k.shape[2]
    out = np.zeros((b, h, sq, d), dtype=np.float32)
    for bi in range(b):
        lk = int(kv_lens[bi]) if kv_lens is not None else sk
        s = q[bi] @ np.swapaxes(k[bi, :, :lk], -1, -2)
        s = s / np.sqrt(d) if not scale else s * scale
        if causal:
            i = np.arange(sq)[:, None]
            t = np.arange(lk)[None, :]
            s = np.where(t > i + (lk - sq), -np.inf, s)
        m = s.max(axis=-1, keepdims=True)
        p = np.exp(s - m)
        p = p / p.sum(axis=-1, keepdims=True)
        out[bi] = (p @ v[bi, :, :lk]).astype(np.float32)
    return out


def attention_flops(b: int, h: int, sq: int, sk: int, d: int, causal: bool = True,
                    kv_lens=None) -> int:
    """Algorithmic FLOPs: 4*D per visible (query, key) pair (QK^T and PV, 2 FLOPs per MAC)."""
    total = 0
    for bi in range(b):
        lk = int(kv_lens[bi]) if kv_lens is not None else sk
        if causal:
            off = lk - sq
            pairs = sum(min(lk, i + off + 1) for i in range(sq))
        else:
            pairs = sq * lk
        total += pairs
    return 4 * d * h * total


__all__ = ["attention", "attention_flops", "attention_head", "attention_head_f64", "attention_np",
           "build",
           "max_threads"]
