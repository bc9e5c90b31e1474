"""The software exp2 used for part of the softmax exponentials (exp2_poly.cuh).

Emulates the device sequence in float32 NumPy -- clamp to -126, round with the
1.5*2^23 magic number, cubic minimax polynomial on r in [-1/2, 1/2], and the
exponent-field add of bits(t) << 23 -- and checks it against exp2 over the
whole range the softmax produces (x <= 0).  Also re-derives the coefficients
with the committed generator.
"""

from __future__ import annotations

import re
import subprocess
import sys

import numpy as np

from conftest import ROOT

HDR = ROOT / "warpforth_b200" / "csrc" / "exp2_poly.cuh"


def _coeffs() -> list[np.float32]:
    text = HDR.read_text()
    return [np.float32(float(re.search(rf"kC{i} = ([-0-9.e]+)f;", text).group(1)))
            for i in range(4)]


def exp2_poly_f32(x: np.ndarray) -> np.ndarray:
    c0, c1, c2, c3 = _coeffs()
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    j = (t - magic).astype(np.float32)
    r = (x - j).astype(np.float32)
    p = (c3 * r + c2).astype(np.float32)
    p = (p * r + c1).astype(np.float32)
    p = (p * r + c0).astype(np.float32)
    bits = p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def test_poly_matches_exp2_on_softmax_range():
    x = np.concatenate([np.linspace(-126.0, 0.0, 2_000_001, dtype=np.float32),
                        -np.random.default_rng(0).exponential(4.0, 200_000).astype(np.float32)])
    x = x[x >= -126.0]
    got = exp2_poly_f32(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(got / ref - 1.0)
    assert rel.max() < 2e-4  # 7.5e-5 from the polynomial + f32 rounding of the steps


def test_poly_clamps_very_negative_inputs_to_tiny_nonnegative_values():
    x = np.array([-127.0, -200.0, -1e6, -3.4e38], dtype=np.float32)
    got = exp2_poly_f32(x)
    assert np.all(got >= 0) and np.all(got < 1e-37)


def test_header_is_what_the_generator_produces():
    gen = ROOT / "warpforth_b200" / "csrc" / "gen_exp2_poly.py"
    out = subprocess.run([sys.executable, str(gen)], capture_output=True, text=True, check=True)
    assert out.stdout == HDR.read_text()
