"""Pins the CPU oracle to the reference's own attention tests (no GPU needed).

The golden cases in tests/golden/attention_kats.json are the inputs of
gpu_test/test_kernels.py:662-875 with the outputs of that file's NumPy
``_attention_reference`` (:651-659); the tolerances are the ones those tests use
(pytest.approx default rel 1e-6 for the f64 kernels, rel 1e-5 for the f32 one).
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

import oracle
from conftest import approx_list


def _case(kats, name):
    c = kats[name]
    s, d = c["seq_len"], c["head_dim"]
    arr = lambda key: np.asarray(c[key], dtype=np.float64).reshape(s, d)  # noqa: E731
    return c, arr("q"), arr("k"), arr("v")


@pytest.mark.parametrize("name", ["test_naive_attention_f64", "test_naive_attention_f64_16x64"])
def test_oracle_f64_io_matches_reference_kats(kats, name):
    c, q, k, v = _case(kats, name)
    out = oracle.attention_head_f64(q, k, v).ravel().tolist()
    assert out == approx_list(c["expected"], rel=c["rel_tol"])


def test_oracle_f32_io_matches_reference_kat(kats):
    c, q, k, v = _case(kats, "test_naive_attention_f32")
    assert c["f32_io"]
    out = oracle.attention_head(q, k, v).ravel().tolist()
    assert out == approx_list(c["expected"], rel=c["rel_tol"])


def test_kat_launch_geometry_is_reference_abi(kats):
    # The reference launches grid=(S,1,1), block=(S,1,1) and reads O (param 3).
    for c in kats.values():
        assert c["grid"] == [c["seq_len"], 1, 1]
        assert c["block"] == [c["seq_len"], 1, 1]
        assert c["output_param"] == 3


def test_oracle_matches_gpt2_head_call_golden(gpt2_head_golden):
    torch = pytest.importorskip("torch")
    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 12, 64, 64) for _ in range(3))
    digest = hashlib.sha256(b"".join(t.numpy().tobytes() for t in (q, k, v))).hexdigest()
    assert digest == str(gpt2_head_golden["input_sha256"]), "torch RNG stream changed"
    out = oracle.attention(q.numpy(), k.numpy(), v.numpy())
    ref = gpt2_head_golden["reference_f64"]
    assert np.abs(out - ref).max() <= 1e-6
    assert np.abs(out - gpt2_head_golden["torch_sdpa_f32"]).max() <= 1e-5


def test_literal_and_strided_oracles_agree_bitwise():
    rng = np.random.default_rng(7)
    for s, d in [(1, 1), (2, 4), (3, 5), (17, 64), (65, 32)]:
        q, k, v = (rng.standard_normal((1, 1, s, d)).astype(np.float32) for _ in range(3))
        lit = oracle.attention_head(q[0, 0], k[0, 0], v[0, 0])
        gen = oracle.attention(q, k, v)[0, 0]
        assert np.array_equal(lit, gen), (s, d)


def test_numpy_and_c_oracles_agree():
    rng = np.random.default_rng(8)
    q, k, v = (rng.standard_normal((2, 3, 40, 64)).astype(np.float32) for _ in range(3))
    assert np.abs(oracle.attention(q, k, v) - oracle.attention_np(q, k, v)).max() < 1e-6
    # non-causal, explicit scale, Sq != Sk, per-batch lengths
    kk, vv = (rng.standard_normal((2, 3, 50, 64)).astype(np.float32) for _ in range(2))
    lens = np.array([50, 45], dtype=np.int32)
    a = oracle.attention(q, kk, vv, scale=0.1, causal=True, kv_lens=lens)
    b = oracle.attention_np(q, kk, vv, scale=0.1, causal=True, kv_lens=lens)
    assert np.abs(a - b).max() < 1e-6


def test_oracle_strided_views_and_ranges():
    rng = np.random.default_rng(9)
    base = rng.standard_normal((2, 33, 4, 3, 32)).astype(np.float32)  # [B, S, H, 3, D]
    q, k, v = (np.transpose(base[:, :, :, i, :], (0, 2, 1, 3)) for i in range(3))
    full = oracle.attention(np.ascontiguousarray(q), np.ascontiguousarray(k),
                            np.ascontiguousarray(v))
    assert np.array_equal(oracle.attention(q, k, v), full)
    part = oracle.attention(q, k, v, bh_range=(3, 6), row_range=(5, 20))
    flat = part.reshape(8, 33, 32)
    assert np.array_equal(flat[3:6, 5:20], full.reshape(8, 33, 32)[3:6, 5:20])
    assert not flat[:3].any() and not flat[6:].any()


def test_oracle_rejects_causal_with_more_queries_than_keys():
    q = np.zeros((1, 1, 4, 8), np.float32)
    k = np.zeros((1, 1, 3, 8), np.float32)
    with pytest.raises(RuntimeError):
        oracle.attention(q, k, k)


def test_flop_counts_match_workload_definitions():
    assert oracle.attention_flops(8, 12, 1024, 1024, 64) == 12_897_484_800
    assert oracle.attention_flops(16, 48, 8192, 8192, 64) == 6_597_875_073_024
    assert oracle.attention_flops(1, 12, 64, 64, 64) == 6_389_760
