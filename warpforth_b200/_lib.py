"""ctypes binding of libwfattn (include/wfattn.h).

The library is loaded from ``warpforth_b200/lib/libwfattn.so`` (built in-tree by
``python -m warpforth_b200.build``).  There is no fallback: if the library is
missing or a call fails, a ``WfattnError`` is raised.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libwfattn.so"

# wfattn_status_t
OK, INVALID_ARG, UNSUPPORTED, CUDA_ERROR, TIMEOUT = range(5)
# wfattn_dtype_t
DTYPE_F32, DTYPE_BF16 = 0, 1

EXPORTED_SYMBOLS = (
    "wfattn_version", "wfattn_status_string", "wfattn_last_error", "wfattn_attention",
    "wfattn_prefill", "wfattn_prefill_gather", "wfattn_prefill_multicast",
    "wfattn_decode_workspace_size", "wfattn_decode",
    "wfattn_decode_f32_workspace_size", "wfattn_decode_f32", "wfattn_decode_noalloc", "wfattn_device_status", "wfattn_peer_alloc", "wfattn_peer_open",
    "wfattn_peer_close", "wfattn_peer_free",
)


class WfattnError(RuntimeError):
    """A libwfattn call returned a status other than WFATTN_OK."""

    def __init__(self, status: int, message: str) -> None:
        super().__init__(f"[{status_name(status)}] {message}")
        self.status = status


class Dim3(ctypes.Structure):
    _fields_ = [("x", ctypes.c_uint), ("y", ctypes.c_uint), ("z", ctypes.c_uint)]


class PeerHandle(ctypes.Structure):
    """wfattn_peer_handle_t: 64 opaque bytes naming a device buffer across processes."""

    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


_lib = None
_i64 = ctypes.c_int64
_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p


def load() -> ctypes.CDLL:
    """Load libwfattn.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise WfattnError(CUDA_ERROR, f"{LIB_PATH} is missing; run `python -m warpforth_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.wfattn_version.restype = ctypes.c_int
    lib.wfattn_status_string.restype = ctypes.c_char_p
    lib.wfattn_status_string.argtypes = [ctypes.c_int]
    lib.wfattn_last_error.restype = ctypes.c_char_p
    lib.wfattn_attention.restype = ctypes.c_int
    lib.wfattn_attention.argtypes = [_vp, _vp, _vp, _vp, _i64, _i64, ctypes.POINTER(Dim3),
                                     ctypes.POINTER(Dim3), _vp]
    lib.wfattn_prefill.restype = ctypes.c_int
    lib.wfattn_prefill.argtypes = [ctypes.c_int, _i64, _i64, _i64, _i64, _i64,
                                   _vp, _i64p, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                                   ctypes.c_float, ctypes.c_int, _vp]
    lib.wfattn_prefill_gather.restype = ctypes.c_int
    lib.wfattn_prefill_gather.argtypes = [_i64, _i64, _i64, _i64, _i64, _vp, _i64p, _vp, _i64p,
                                          _vp, _i64p, ctypes.POINTER(_vp), ctypes.c_int, _i64p,
                                          ctypes.c_float, ctypes.c_int, _vp]
    lib.wfattn_prefill_multicast.restype = ctypes.c_int
    lib.wfattn_prefill_multicast.argtypes = lib.wfattn_prefill.argtypes[1:]
    lib.wfattn_decode_workspace_size.restype = ctypes.c_size_t
    lib.wfattn_decode_workspace_size.argtypes = [_i64, _i64, _i64, _i64]
    lib.wfattn_decode.restype = ctypes.c_int
    lib.wfattn_decode.argtypes = [_i64, _i64, _i64, _i64, _vp, _i64p, _vp, _i64p, _vp, _i64p,
                                  _vp, _vp, _i64p, ctypes.c_float, _vp, ctypes.c_size_t, _vp]
    lib.wfattn_decode_f32_workspace_size.restype = ctypes.c_size_t
    lib.wfattn_decode_f32_workspace_size.argtypes = [_i64, _i64, _i64, _i64]
    lib.wfattn_decode_f32.restype = ctypes.c_int
    lib.wfattn_decode_f32.argtypes = lib.wfattn_decode.argtypes
    lib.wfattn_decode_noalloc.restype = ctypes.c_int
    lib.wfattn_decode_noalloc.argtypes = [_i64, _i64, _i64, _i64, _vp, _i64p, _vp, _i64p, _vp,
                                          _i64p, _vp, _vp, _i64p, ctypes.c_float, _vp]
    lib.wfattn_device_status.restype = ctypes.c_int
    lib.wfattn_device_status.argtypes = [_vp, ctypes.c_int]
    lib.wfattn_peer_alloc.restype = ctypes.c_int
    lib.wfattn_peer_alloc.argtypes = [ctypes.c_size_t, ctypes.c_int, ctypes.POINTER(_vp),
                                      ctypes.POINTER(PeerHandle)]
    lib.wfattn_peer_open.restype = ctypes.c_int
    lib.wfattn_peer_open.argtypes = [ctypes.POINTER(PeerHandle), ctypes.c_int, ctypes.POINTER(_vp)]
    lib.wfattn_peer_close.restype = ctypes.c_int
    lib.wfattn_peer_close.argtypes = [_vp, ctypes.c_int]
    lib.wfattn_peer_free.restype = ctypes.c_int
    lib.wfattn_peer_free.argtypes = [_vp, ctypes.c_int]
    _lib = lib
    return lib


def status_name(status: int) -> str:
    names = {OK: "WFATTN_OK", INVALID_ARG: "WFATTN_INVALID_ARG", UNSUPPORTED: "WFATTN_UNSUPPORTED",
             CUDA_ERROR: "WFATTN_CUDA_ERROR", TIMEOUT: "WFATTN_TIMEOUT"}
    return names.get(status, f"status {status}")


def check(status: int) -> None:
    """Raise WfattnError with the library's message unless status is WFATTN_OK."""
    if status != OK:
        msg = load().wfattn_last_error().decode(errors="replace")
        raise WfattnError(status, msg)


def strides_arg(strides) -> ctypes.Array | None:
    if strides is None:
        return None
    arr = (ctypes.c_int64 * 3)(*[int(s) for s in strides] + [0] * (3 - len(strides)))
    return arr
