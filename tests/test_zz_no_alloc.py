"""wfattn_decode_noalloc: decode for callers that cannot allocate device memory.

Some callers only hold the buffers they were handed -- a plugin whose host
framework owns every byte of device memory through its own pool, or a caller
reaching the library through a foreign-function interface with no CUDA
allocator of its own -- so they cannot provide the decode workspace.  This
entry point keeps the split-KV partials in a static 8 MiB device array inside
the library instead.  The GPU test calls it through the C ABI twice in a row
(the array keeps the previous call's contents) and compares each result with
the workspace-based wfattn_decode bit for bit: both run the same kernels in the
same order on the same inputs, only the scratch address differs.  This file
sorts last so that a run stopping at the first failure has run everything
else first.
"""

from __future__ import annotations

import ctypes

import pytest

from warpforth_b200 import _lib


def test_noalloc_rejects_shapes_beyond_the_static_scratch():
    lib = _lib.load()
    # 64 * 25 * ceil(8192 / 256) = 51,200 chunk partials > 31,775: rejected on the host
    st = lib.wfattn_decode_noalloc(64, 25, 64, 8192, 16, None, 16, None, 16, None, 16, 16, None,
                                   0.0, None)
    assert st == _lib.INVALID_ARG
    assert b"static scratch" in lib.wfattn_last_error()


@pytest.mark.gpu
def test_noalloc_decode_matches_workspace_decode_twice():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from warpforth_b200 import warpforth as wf

    dev = torch.device("cuda", 0)
    lib = _lib.load()
    cases = [((1, 300, 513, 4096), 3, 4096), ((257, 1, 2000), 5, 2048)]
    for lens, heads, lmax in cases:
        g = torch.Generator().manual_seed(len(lens))
        b = len(lens)
        q = torch.randn(b, heads, 64, generator=g).bfloat16().to(dev)
        kc = torch.randn(b, heads, lmax, 64, generator=g).bfloat16().to(dev)
        vc = torch.randn(b, heads, lmax, 64, generator=g).bfloat16().to(dev)
        kl = torch.tensor(lens, dtype=torch.int32, device=dev)
        ref = wf.decode(q, kc, vc, kl)
        assert torch.isfinite(ref).all()
        for _ in range(2):  # the second call finds the first call's partials in the array
            out = torch.full((b, heads, 64), float("nan"), device=dev)
            st = lib.wfattn_decode_noalloc(
                b, heads, 64, lmax, q.data_ptr(), None, kc.data_ptr(), None, vc.data_ptr(), None,
                kl.data_ptr(), out.data_ptr(), None, ctypes.c_float(0.0),
                torch.cuda.current_stream(dev).cuda_stream)
            _lib.check(st)
            assert torch.equal(out, ref)
    wf.device_status(clear=True)
