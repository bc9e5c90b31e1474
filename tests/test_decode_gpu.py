"""GPU parity of the split-KV decode kernel against the CPU oracle.

Decode is the single-query case of the oracle's batched form: query row 0
against the first kv_lens[b] keys of each (batch, head) of a padded cache.
Tolerance: max|o - ref| / max|ref| per (batch, head) <= 2e-2 (bf16 inputs,
f32 accumulation), ref = f64 oracle on the same bf16 values.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

BF16_REL_TOL = 2e-2


@pytest.fixture(scope="module")
def wf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from warpforth_b200 import warpforth

    return warpforth


def _ref(q, kc, vc, lens, scale=None):
    # q [B, H, D] -> [B, H, 1, D]; causal off (the single query sees every valid key)
    return oracle.attention(q.float().numpy()[:, :, None, :], kc.float().numpy(),
                            vc.float().numpy(), causal=False, kv_lens=lens.numpy(),
                            scale=scale)[:, :, 0, :]


def _rel(out, ref):
    b, h = ref.shape[:2]
    o = out.reshape(b * h, -1)
    r = ref.reshape(b * h, -1)
    return float((np.abs(o - r).max(axis=1) / np.abs(r).max(axis=1)).max())


def _case(b, h, lmax, lens, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, 64, generator=g).bfloat16()
    kc = torch.randn(b, h, lmax, 64, generator=g).bfloat16()
    vc = torch.randn(b, h, lmax, 64, generator=g).bfloat16()
    return q, kc, vc, torch.tensor(lens, dtype=torch.int32)


@pytest.mark.parametrize("lens", [[1], [2], [255], [256], [257], [511, 512, 513, 1000],
                                  [1, 4096, 17, 3000]])
def test_decode_ragged_lengths(wf, lens):
    lmax = max(lens)
    q, kc, vc, kl = _case(len(lens), 3, lmax, lens, 11)
    out = wf.decode(q.cuda(), kc.cuda(), vc.cuda(), kl.cuda()).cpu().numpy()
    assert np.isfinite(out).all()
    assert _rel(out, _ref(q, kc, vc, kl)) <= BF16_REL_TOL


def test_decode_many_batches_unplanned_order(wf):
    # more batches than the kernel orders by length in shared memory (1024):
    # the work items are then enumerated chunk-major with empty chunks skipped
    b = 1100
    lens = torch.randint(1, 301, (b,), generator=torch.Generator().manual_seed(15),
                         dtype=torch.int32).tolist()
    q, kc, vc, kl = _case(b, 1, 300, lens, 14)
    out = wf.decode(q.cuda(), kc.cuda(), vc.cuda(), kl.cuda()).cpu().numpy()
    assert np.isfinite(out).all()
    sel = list(range(0, 40)) + list(range(b - 40, b))
    assert _rel(out[sel], _ref(q[sel], kc[sel], vc[sel], kl[sel])) <= BF16_REL_TOL


def test_decode_padding_is_never_read(wf):
    # NaN in the padding past kv_lens must not reach the output
    q, kc, vc, kl = _case(2, 2, 600, [300, 512], 12)
    kcn, vcn = kc.clone(), vc.clone()
    for b, L in enumerate(kl.tolist()):
        kcn[b, :, L:] = float("nan")
        vcn[b, :, L:] = float("nan")
    out = wf.decode(q.cuda(), kcn.cuda(), vcn.cuda(), kl.cuda()).cpu().numpy()
    assert np.isfinite(out).all()
    assert _rel(out, _ref(q, kc, vc, kl)) <= BF16_REL_TOL


def test_decode_strided_query_scale_and_workspace_reuse(wf):
    q4, kc, vc, kl = _case(4, 5, 700, [700, 1, 350, 699], 13)
    qs = torch.zeros(4, 5, 2, 64, dtype=torch.bfloat16)
    qs[:, :, 1] = q4
    ws = wf.DecodeWorkspace()
    for scale in (None, 0.3):
        out = wf.decode(qs.cuda()[:, :, 1], kc.cuda(), vc.cuda(), kl.cuda(), scale=scale,
                        workspace=ws).cpu().numpy()
        assert _rel(out, _ref(q4, kc, vc, kl, scale=scale)) <= BF16_REL_TOL


def test_decode_config4_shape(wf):
    # B=64, H=25, D=64, kv_lens ~ U[512, 4096] from seed 3, cache from seed 3 after the lengths
    lens = torch.randint(512, 4097, (64,), generator=torch.Generator().manual_seed(3),
                         dtype=torch.int64).to(torch.int32)
    assert int(lens.sum()) == 142_652 and int(lens.min()) == 526 and int(lens.max()) == 4038
    torch.manual_seed(3)
    kc = torch.randn(64, 25, 4096, 64, dtype=torch.bfloat16)
    vc = torch.randn(64, 25, 4096, 64, dtype=torch.bfloat16)
    q = torch.randn(64, 25, 64, dtype=torch.bfloat16)
    out = wf.decode(q.cuda(), kc.cuda(), vc.cuda(), lens.cuda()).cpu().numpy()
    # all 64 sequences x 25 heads against the f64 oracle (under 1 GFLOP)
    assert np.isfinite(out).all()
    assert _rel(out, _ref(q, kc, vc, lens)) <= BF16_REL_TOL
    wf.device_status(clear=True)


def test_decode_bad_length_is_reported(wf):
    q, kc, vc, _ = _case(1, 1, 64, [64], 14)
    bad = torch.tensor([65], dtype=torch.int32)
    wf.decode(q.cuda(), kc.cuda(), vc.cuda(), bad.cuda())
    from warpforth_b200 import _lib

    with pytest.raises(_lib.WfattnError, match="kv_lens"):
        wf.device_status(clear=True)
    wf.device_status(clear=True)  # cleared


# ---------------------------------------------------------------- f32 cache (wfattn_decode_f32)
F32_ABS_TOL = 1e-5


def _case_f32(b, h, lmax, lens, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, 64, generator=g)
    kc = torch.randn(b, h, lmax, 64, generator=g)
    vc = torch.randn(b, h, lmax, 64, generator=g)
    return q, kc, vc, torch.tensor(lens, dtype=torch.int32)


@pytest.mark.parametrize("lens", [[1], [2], [127], [128], [129], [255, 256, 257, 1000],
                                  [1, 4096, 17, 3000], [32, 159]])
def test_decode_f32_ragged_lengths_at_the_f32_contract(wf, lens):
    # 128-key chunks: lengths around one and two chunks, a long and a 1-key sequence
    q, kc, vc, kl = _case_f32(len(lens), 3, max(lens), lens, 21)
    out = wf.decode(q.cuda(), kc.cuda(), vc.cuda(), kl.cuda()).cpu().numpy()
    assert np.isfinite(out).all()
    assert np.abs(out - _ref(q, kc, vc, kl)).max() <= F32_ABS_TOL


def test_decode_f32_strided_query_scale_padding_and_gpt2_layout(wf):
    # q as the [B, H, 1, D] view of a [B, 1, H, D] projection (GPT-2's layout), NaN in the
    # cache padding, an explicit scale, and a workspace reused across calls
    q, kc, vc, kl = _case_f32(2, 12, 300, [159, 300], 22)
    qv = q[:, None].contiguous().transpose(1, 2)  # [B, H, 1, D] with strides (H*D, D, H*D, 1)
    kcn, vcn = kc.clone(), vc.clone()
    kcn[0, :, 159:] = float("nan")
    vcn[0, :, 159:] = float("nan")
    ws = wf.DecodeWorkspace()
    for scale in (None, 0.125, 0.3):
        out = wf.decode(qv.cuda(), kcn.cuda(), vcn.cuda(), kl.cuda(), scale=scale,
                        workspace=ws).cpu().numpy()
        assert np.isfinite(out).all()
        assert np.abs(out - _ref(q, kc, vc, kl, scale=scale)).max() <= F32_ABS_TOL


def test_decode_f32_config4_shape(wf):
    # config 4's lengths and shape with an f32 cache (every sequence against the oracle)
    lens = torch.randint(512, 4097, (64,), generator=torch.Generator().manual_seed(3),
                         dtype=torch.int64).to(torch.int32)
    torch.manual_seed(3)
    kc = torch.randn(64, 25, 4096, 64)
    vc = torch.randn(64, 25, 4096, 64)
    q = torch.randn(64, 25, 64)
    out = wf.decode(q.cuda(), kc.cuda(), vc.cuda(), lens.cuda()).cpu().numpy()
    assert np.isfinite(out).all()
    assert np.abs(out - _ref(q, kc, vc, lens)).max() <= F32_ABS_TOL
    wf.device_status(clear=True)


def test_decode_rejects_mixed_dtypes(wf):
    q, kc, vc, kl = _case_f32(1, 1, 8, [8], 23)
    with pytest.raises(ValueError, match="all bfloat16 or all float32"):
        wf.decode(q.cuda(), kc.cuda().bfloat16(), vc.cuda(), kl.cuda())
