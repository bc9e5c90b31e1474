"""wfattn-runner: the warpforth-runner command line with a libwfattn launch path.

CPU tests cover the argument handling (errors exit 1 before any CUDA call, as
in tools/warpforth-runner/warpforth-runner.cpp:93-199,255-283).  GPU tests run
the reference's attention test cases through the runner exactly as its harness
builds the command line (gpu_test/conftest.py:443-483): packed f32 in i64[]
arrays for the f32 kernel, f64[] arrays for the f64 twin.
"""

from __future__ import annotations

import struct
import subprocess

import numpy as np
import pytest

from conftest import ROOT, approx_list

RUNNER = ROOT / "warpforth_b200" / "lib" / "wfattn-runner"


def _run(*args: str) -> subprocess.CompletedProcess:
    if not RUNNER.exists():
        pytest.skip("wfattn-runner not built")
    return subprocess.run([str(RUNNER), *args], capture_output=True, text=True, timeout=120)


@pytest.mark.parametrize("args, needle", [
    ((), "--kernel NAME is required"),
    (("--kernel", "attention"), "at least one --param"),
    (("--kernel", "attention", "--param", "i64:3"), "is a scalar"),
    (("--kernel", "attention", "--param", "i64[]:1", "--output-param", "4"), "out of range"),
    (("--kernel", "attention", "--param", "x64:1"), "unsupported --param type"),
    (("--kernel", "attention", "--param", "i64:1,2", "--output-param", "0"), "one value"),
    (("--kernel", "attention", "--param", "i64[]:1,zz"), "not an integer"),
    (("--kernel", "attention", "--param", "f64[]:1.5,q"), "not a number"),
    (("--kernel", "attention", "--param", "i64[]:1", "--grid", "1,2"), "expects X,Y,Z"),
    (("--kernel", "attention", "--param", "i64[]:1", "--bogus"), "unknown option"),
    (("--kernel", "attention", "--param", "i64[]:1", "--grid"), "requires a value"),
    (("--kernel", "attention", "--param", "i64[]:1"), "takes Q K V O arrays"),
    (("--kernel", "other", "--param", "i64[]:1"), "PTX file is required"),
    (("--kernel", "attention", "--impl", "gpu", "--param", "i64[]:1"), "--impl must be"),
])
def test_runner_argument_errors(args, needle):
    res = _run(*args)
    assert res.returncode == 1
    assert needle in res.stderr


def _pack(values) -> str:
    b = np.asarray(values, dtype=np.float32).tobytes()
    b += b"\x00" * ((8 - len(b) % 8) % 8)
    return ",".join(str(struct.unpack("<q", b[i:i + 8])[0]) for i in range(0, len(b), 8))


def _unpack(csv: str, count: int) -> list[float]:
    raw = b"".join(struct.pack("<q", int(x)) for x in csv.strip().split(","))
    return np.frombuffer(raw, dtype=np.float32)[:count].tolist()


@pytest.mark.gpu
def test_runner_f32_kat_packed_i64(kats):
    c = kats["test_naive_attention_f32"]
    s, d = c["seq_len"], c["head_dim"]
    n = s * d
    n_i64 = (n + 1) // 2
    zeros = ",".join(["0"] * n_i64)
    res = _run("--kernel", "attention",
               "--param", f"i64[]:{_pack(c['q'])}", "--param", f"i64[]:{_pack(c['k'])}",
               "--param", f"i64[]:{_pack(c['v'])}", "--param", f"i64[]:{zeros}",
               "--param", f"i64:{s}", "--param", f"i64:{d}",
               "--grid", f"{s},1,1", "--block", f"{s},1,1",
               "--output-param", "3", "--output-count", str(n_i64))
    assert res.returncode == 0, res.stderr
    assert _unpack(res.stdout, n) == approx_list(c["expected"], rel=c["rel_tol"])


@pytest.mark.gpu
def test_runner_f64_twin_kat(kats):
    c = kats["test_naive_attention_f64_16x64"]
    s, d = c["seq_len"], c["head_dim"]
    n = s * d
    arr = lambda xs: ",".join(repr(float(x)) for x in xs)  # noqa: E731
    res = _run("--kernel", "attention",
               "--param", f"f64[]:{arr(c['q'])}", "--param", f"f64[]:{arr(c['k'])}",
               "--param", f"f64[]:{arr(c['v'])}", "--param", f"f64[]:{arr([0.0] * n)}",
               "--param", f"i64:{s}", "--param", f"i64:{d}",
               "--grid", f"{s},1,1", "--block", f"{s},1,1", "--output-param", "3",
               "--output-count", str(n))
    assert res.returncode == 0, res.stderr
    out = np.array([float(x) for x in res.stdout.strip().split(",")])
    # f32 arithmetic on f32-rounded inputs: the f32 contract, 1e-5 absolute
    assert np.abs(out - np.asarray(c["expected"])).max() <= 1e-5


@pytest.mark.gpu
def test_runner_rejects_foreign_geometry():
    res = _run("--kernel", "attention", "--param", "i64[]:0,0", "--param", "i64[]:0,0",
               "--param", "i64[]:0,0", "--param", "i64[]:0,0", "--param", "i64:2",
               "--param", "i64:2", "--grid", "3,1,1", "--block", "2,1,1", "--output-param", "3")
    assert res.returncode == 1
    assert "WFATTN" in res.stderr.upper() or "grid" in res.stderr
