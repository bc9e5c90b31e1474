"""C-ABI checks that need no GPU: the library loads, exports every symbol that
include/wfattn.h declares, and rejects bad arguments on the host before any
CUDA call (the reference's runner exits on such input instead:
tools/warpforth-runner/warpforth-runner.cpp:93-199,255-283)."""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT
from warpforth_b200 import _lib


def _declared_symbols() -> list[str]:
    text = (ROOT / "include" / "wfattn.h").read_text()
    return re.findall(r"WFATTN_API\s+[\w\s\*]*?\b(wfattn_\w+)\s*\(", text)


def test_header_declares_the_bound_symbols():
    assert sorted(_declared_symbols()) == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared_symbols():
        assert hasattr(lib, name), name


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.wfattn_version() >= 100
    for st in range(5):
        assert lib.wfattn_status_string(st)
    assert lib.wfattn_status_string(99) == b"unknown status"


def _prefill(lib, **kw):
    args = dict(dtype=_lib.DTYPE_F32, b=1, h=1, sq=4, sk=4, d=4, q=16, k=16, v=16, o=16,
                scale=0.0, causal=1)
    args.update(kw)
    return lib.wfattn_prefill(args["dtype"], args["b"], args["h"], args["sq"], args["sk"],
                              args["d"], args["q"], None, args["k"], None, args["v"], None,
                              args["o"], None, args["scale"], args["causal"], None)


@pytest.mark.parametrize("kw", [
    {"q": None}, {"o": None}, {"b": 0}, {"sq": 0}, {"d": 0}, {"sk": 3, "sq": 4},
    {"scale": float("nan")},
])
def test_prefill_rejects_bad_arguments_on_host(kw):
    lib = _lib.load()
    assert _prefill(lib, **kw) == _lib.INVALID_ARG
    assert lib.wfattn_last_error()


def test_prefill_gather_rejects_bad_arguments_on_host():
    lib = _lib.load()
    outs = (ctypes.c_void_p * 9)(*([16] * 9))

    def call(outputs, n, q=16, sq=4, sk=4):
        return lib.wfattn_prefill_gather(1, 1, sq, sk, 64, q, None, 16, None, 16, None,
                                         outputs, n, None, 0.0, 1, None)

    assert call(outs, 0) == _lib.INVALID_ARG
    assert call(outs, 9) == _lib.INVALID_ARG  # at most 8 destinations
    assert call(None, 2) == _lib.INVALID_ARG
    assert call(outs, 2, q=None) == _lib.INVALID_ARG
    assert call(outs, 2, sq=5, sk=4) == _lib.INVALID_ARG  # causal needs seq_k >= seq_q
    assert lib.wfattn_last_error()


def test_reference_abi_rejects_foreign_geometry_on_host():
    lib = _lib.load()
    bad = _lib.Dim3(3, 1, 1)
    good = _lib.Dim3(4, 1, 1)
    st = lib.wfattn_attention(16, 16, 16, 16, 4, 4, ctypes.byref(bad), ctypes.byref(good), None)
    assert st == _lib.INVALID_ARG
    assert b"grid" in lib.wfattn_last_error()
    st = lib.wfattn_attention(16, 16, 16, 16, 4, 4, ctypes.byref(good), ctypes.byref(bad), None)
    assert st == _lib.INVALID_ARG
    assert lib.wfattn_attention(16, 16, 16, 16, 0, 4, None, None, None) == _lib.INVALID_ARG


def test_decode_rejects_bad_arguments_on_host():
    lib = _lib.load()
    ws = lib.wfattn_decode_workspace_size(2, 3, 1000, 64)
    assert ws == 2 * 3 * 4 * 66 * 4
    assert lib.wfattn_decode_workspace_size(0, 3, 1000, 64) == 0
    # missing workspace
    st = lib.wfattn_decode(2, 3, 64, 1000, 16, None, 16, None, 16, None, 16, 16, None, 0.0,
                           None, 0, None)
    assert st == _lib.INVALID_ARG
    # unsupported head_dim
    st = lib.wfattn_decode(2, 3, 32, 1000, 16, None, 16, None, 16, None, 16, 16, None, 0.0,
                           16, 1 << 20, None)
    assert st == _lib.UNSUPPORTED


def test_check_raises_with_library_message():
    lib = _lib.load()
    with pytest.raises(_lib.WfattnError, match="INVALID_ARG"):
        _lib.check(_prefill(lib, b=0))


def _integration_blocks(lang: str) -> list[str]:
    return re.findall(rf"```{lang}\n(.*?)```", (ROOT / "INTEGRATION.md").read_text(), re.S)


def test_integration_c_examples_compile(tmp_path):
    """The multi-GPU C examples (multicast: wfattn_prefill_multicast; peer buffers:
    wfattn_prefill_gather) compile as written."""
    import shutil
    import subprocess

    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    blocks = _integration_blocks("c")
    assert len(blocks) == 2
    for i, block in enumerate(blocks):
        src = tmp_path / f"example{i}.c"
        src.write_text(
            "#include <stdint.h>\n#include \"wfattn.h\"\n"
            "void step(int64_t B, int64_t H, int64_t S, int G, int rank, int dev, void *mc,\n"
            "          int slot, const void *q_local, const int64_t *q_strides,\n"
            "          const void *k_local, const int64_t *k_strides, const void *v_local,\n"
            "          const int64_t *v_strides, void *stream) {\n" + block + "}\n")
        res = subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-Wno-unused-result", "-c",
                              "-I", str(ROOT / "include"), str(src),
                              "-o", str(tmp_path / f"e{i}.o")], capture_output=True, text=True)
        assert res.returncode == 0, res.stderr


def test_integration_python_binding_reports_errors():
    """The ctypes binding shown for demo/warpforth.py loads the library and surfaces its
    error text (a host-side argument error; no GPU call is made)."""
    block = _integration_blocks("python")[0]
    ns: dict = {}
    exec(block.replace('"warpforth_b200/lib/libwfattn.so"', repr(str(_lib.LIB_PATH))), ns)
    lib = ns["lib"]
    assert lib.wfattn_attention(None, None, None, None, 4, 4, None, None, None) == _lib.INVALID_ARG
    assert "null" in lib.wfattn_last_error().decode()


def test_decode_shape_bounds_are_checked_without_overflow():
    """batch*heads and max_kv_len are bounded on the host, so a huge shape can neither wrap
    the workspace size to a small number nor reach a launch (no GPU call is made)."""
    lib = _lib.load()
    assert lib.wfattn_decode_workspace_size(64, 25, 4096, 64) == 64 * 25 * 16 * 66 * 4
    huge = 1 << 62
    assert lib.wfattn_decode_workspace_size(huge, huge, 4096, 64) == 0
    assert lib.wfattn_decode_workspace_size(1 << 31, 1, 4096, 64) == 0
    assert lib.wfattn_decode_workspace_size(1, 1, 1 << 31, 64) == 0
    for b, h, lmax in ((huge, huge, 4096), (1 << 31, 1, 256), (1, 1, 1 << 40)):
        st = lib.wfattn_decode(b, h, 64, lmax, 16, None, 16, None, 16, None, 16, 16, None, 0.0,
                               16, 1 << 40, None)
        assert st == _lib.INVALID_ARG
        assert b"2^31-1" in lib.wfattn_last_error()
        st = lib.wfattn_decode_noalloc(b, h, 64, lmax, 16, None, 16, None, 16, None, 16, 16,
                                       None, 0.0, None)
        assert st == _lib.INVALID_ARG
        assert b"2^31-1" in lib.wfattn_last_error()


def test_f32_decode_workspace_is_sized_for_128_key_chunks():
    lib = _lib.load()
    # 128-key chunks for an f32 cache: twice the partials of the bf16 decode's 256-key chunks
    assert lib.wfattn_decode_f32_workspace_size(64, 25, 4096, 64) == 64 * 25 * 32 * 66 * 4
    assert lib.wfattn_decode_f32_workspace_size(1, 12, 159, 64) == 12 * 2 * 66 * 4
    assert lib.wfattn_decode_f32_workspace_size(1 << 40, 1 << 40, 4096, 64) == 0
    st = lib.wfattn_decode_f32(1, 1, 64, 64, 16, None, 16, None, 16, None, 16, 16, None, 0.0,
                               16, 100, None)
    assert st == _lib.INVALID_ARG  # workspace too small: rejected on the host
    assert b"workspace" in lib.wfattn_last_error()
