"""The reference's own compiled attention kernel, run as an opaque arm -- TEST INFRASTRUCTURE ONLY.

WarpForth ships its attention kernel compiled: ``demo/attention.ptx`` is what
``warpforthc demo/attention.forth`` produced (demo/README.md:14-20).  The
reference runs it two ways: PyCUDA ``module_from_buffer`` +
``get_function("attention")`` launched with grid = block = (S, 1, 1)
(demo/warpforth.py:26-49), and the runner's ``cuModuleLoadData`` +
``cuLaunchKernel`` (tools/warpforth-runner/warpforth-runner.cpp:297-321).
``ReferencePtxKernel`` does the same through the CUDA driver API with ctypes
(PyCUDA is not installed), on torch's primary context and current stream.

The file is copied byte for byte into ``oracle/_ref/attention.ptx`` by
``make -C oracle ref`` (git-ignored; it travels with the tree to the GPU
machine).  Its bytes are handed straight to the driver: nothing here prints,
parses or searches them.

Valid domain, from the kernel's source (demo/attention.forth): 2 <= S <= 1024.
Its max loop ``SEQ_LEN 1 DO`` is post-test (lib/Translation/ForthToMLIR/
ForthToMLIR.cpp:1081-1085), so S = 1 never terminates; S > 1024 overruns its
shared ``f64[1024]`` score array and the block-size limit.  Both are refused
here before any launch.

Only ``tests/`` and ``bench.py``'s reference legs use this module; the library
(``warpforth_b200``) never does.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

PTX_PATH = Path(__file__).resolve().parent / "_ref" / "attention.ptx"
MIN_SEQ, MAX_SEQ = 2, 1024

_CU_SUCCESS = 0


class ReferencePtxError(RuntimeError):
    """A driver call on the reference kernel failed, or its inputs are outside its domain."""


def available() -> bool:
    return PTX_PATH.exists()


class _Driver:
    def __init__(self) -> None:
        self.lib = ctypes.CDLL("libcuda.so.1")
        self.lib.cuGetErrorString.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p)]

    def check(self, rc: int, what: str) -> None:
        if rc != _CU_SUCCESS:
            msg = ctypes.c_char_p()
            self.lib.cuGetErrorString(rc, ctypes.byref(msg))
            text = msg.value.decode() if msg.value else f"error {rc}"
            raise ReferencePtxError(f"{what}: {text}")


class ReferencePtxKernel:
    """``attention(Q, K, V, O, SEQ_LEN, HEAD_DIM)`` from the reference's compiled PTX.

    Same call as the reference's PyCUDA wrapper: ``kernel(q, k, v, o, seq_len,
    head_dim)`` on contiguous f32 CUDA tensors of one head ([S, D]); ``o`` is
    overwritten.  Asynchronous on torch's current stream.
    """

    def __init__(self, ptx_path: str | Path = PTX_PATH) -> None:
        import torch

        path = Path(ptx_path)
        if not path.exists():
            raise ReferencePtxError(f"{path} is missing; run `make -C oracle ref` where the "
                                    f"reference tree is present")
        torch.cuda.init()
        torch.empty(1, device="cuda")  # the runtime makes the primary context current
        self._drv = _Driver()
        lib = self._drv.lib
        ctx = ctypes.c_void_p()
        self._drv.check(lib.cuCtxGetCurrent(ctypes.byref(ctx)), "cuCtxGetCurrent")
        if not ctx.value:
            raise ReferencePtxError("no current CUDA context")
        self._image = path.read_bytes() + b"\0"  # kept alive while the module is loaded
        self._module = ctypes.c_void_p()
        self._drv.check(lib.cuModuleLoadData(ctypes.byref(self._module),
                                             ctypes.c_char_p(self._image)), "cuModuleLoadData")
        self._fn = ctypes.c_void_p()
        self._drv.check(lib.cuModuleGetFunction(ctypes.byref(self._fn), self._module,
                                                b"attention"), "cuModuleGetFunction")
        lib.cuLaunchKernel.argtypes = [
            ctypes.c_void_p, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, ctypes.c_uint,
            ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, ctypes.c_void_p,
            ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)]

    def __call__(self, q, k, v, o, seq_len: int, head_dim: int) -> None:
        import torch

        s, d = int(seq_len), int(head_dim)
        if not MIN_SEQ <= s <= MAX_SEQ:
            raise ReferencePtxError(f"the reference kernel is valid for {MIN_SEQ} <= SEQ_LEN <= "
                                    f"{MAX_SEQ}, got {s}")
        if d < 1:
            raise ReferencePtxError(f"HEAD_DIM must be >= 1, got {d}")
        for name, t in (("q", q), ("k", k), ("v", v), ("o", o)):
            if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
                    and t.numel() >= s * d):
                raise ReferencePtxError(f"{name} must be a contiguous f32 CUDA tensor of at "
                                        f"least SEQ_LEN*HEAD_DIM elements")
        # kernel parameters in the reference's order: four bare device pointers, then
        # SEQ_LEN and HEAD_DIM as i64 (warpforth-runner.cpp:313-315)
        vals = [ctypes.c_uint64(t.data_ptr()) for t in (q, k, v, o)]
        vals += [ctypes.c_int64(s), ctypes.c_int64(d)]
        params = (ctypes.c_void_p * 6)(*[ctypes.cast(ctypes.byref(x), ctypes.c_void_p)
                                          for x in vals])
        stream = torch.cuda.current_stream(q.device).cuda_stream
        self._drv.check(self._drv.lib.cuLaunchKernel(self._fn, s, 1, 1, s, 1, 1, 0, stream,
                                                     params, None), "cuLaunchKernel")


def make_reference_eager_attn(kernel: ReferencePtxKernel):
    """The demo's GPT-2 attention patch around the reference kernel (demo/gpt2_generate.py:25-54):
    contiguous copies of q/k/v, a zeroed output, one launch per head of batch entry 0, the
    output returned as [B, S, H, D]; mask, dropout and scaling arguments are not used."""
    import torch

    def reference_eager_attn(module, query, key, value, attention_mask=None, **kwargs):
        seq_len, head_dim = query.shape[2], query.shape[3]
        q, k, v = query.contiguous(), key.contiguous(), value.contiguous()
        out = torch.zeros_like(q)
        for h in range(q.shape[1]):
            kernel(q[0, h], k[0, h], v[0, h], out[0, h], seq_len, head_dim)
        return out.transpose(1, 2), None

    return reference_eager_attn
