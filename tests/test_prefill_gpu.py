"""GPU parity of the prefill kernels against the CPU oracle and the reference's goldens.

f32 path (the drop-in for demo/attention.forth): max abs error <= 1e-5 against
the f64 oracle on the same f32 inputs, and the reference's own attention tests
(gpu_test/test_kernels.py:662-875) at their tolerances.
bf16 path (tcgen05 kernel): per (batch, head), max|o - ref| / max|ref| <= 2e-2
with ref = the f64 oracle on the same bf16-rounded inputs.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import approx_list

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F32_ABS_TOL = 1e-5
BF16_REL_TOL = 2e-2


@pytest.fixture(scope="module")
def wf():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from warpforth_b200 import warpforth

    return warpforth


def _randn(shape, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


def _oracle(q, k, v, **kw):
    return oracle.attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), **kw)


def _bf16_rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    b, h = ref.shape[:2]
    o = out.reshape(b * h, -1)
    r = ref.reshape(b * h, -1)
    return float((np.abs(o - r).max(axis=1) / np.abs(r).max(axis=1)).max())


# ---------------------------------------------------------------- reference ABI
@pytest.mark.parametrize("name", ["test_naive_attention_f32", "test_naive_attention_f64",
                                  "test_naive_attention_f64_16x64"])
def test_reference_kats_through_attention_kernel(wf, kats, name):
    c = kats[name]
    s, d = c["seq_len"], c["head_dim"]
    q, k, v = (torch.tensor(c[x], dtype=torch.float32).reshape(s, d).cuda() for x in "qkv")
    o = torch.full_like(q, float("nan"))
    wf.AttentionKernel()(q, k, v, o, s, d)
    out = o.cpu().numpy().ravel()
    assert np.isfinite(out).all()
    if c["f32_io"]:
        assert out.tolist() == approx_list(c["expected"], rel=c["rel_tol"])
    else:
        # f64 test twins: inputs rounded to f32 here, so compare at the f32 contract
        assert np.abs(out - np.asarray(c["expected"])).max() <= F32_ABS_TOL
    ref = oracle.attention_head(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()).ravel()
    assert np.abs(out - ref).max() <= F32_ABS_TOL


def test_gpt2_head_call_golden(wf, gpt2_head_golden):
    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 12, 64, 64) for _ in range(3))
    # one launch per head through the reference-shaped ABI ...
    o = torch.empty(1, 12, 64, 64, device="cuda")
    kern = wf.AttentionKernel()
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    for h in range(12):
        kern(qc[0, h], kc[0, h], vc[0, h], o[0, h], 64, 64)
    # ... and all heads in one batched launch
    ob = wf.attention(qc, kc, vc)
    for out in (o, ob):
        out = out.cpu().numpy()
        assert np.abs(out - gpt2_head_golden["reference_f64"]).max() <= F32_ABS_TOL
        assert np.abs(out - gpt2_head_golden["torch_sdpa_f32"]).max() <= F32_ABS_TOL


# ---------------------------------------------------------------- f32 sweeps
@pytest.mark.parametrize("s", [1, 2, 3, 17, 63, 64, 65, 127, 128, 129, 1024, 1500])
@pytest.mark.parametrize("d", [4, 64])
def test_f32_single_head_sizes(wf, s, d):
    q, k, v = (_randn((1, 1, s, d), 100 + i) for i in range(3))
    out = wf.attention(q.cuda(), k.cuda(), v.cuda()).cpu().numpy()
    assert np.abs(out - _oracle(q, k, v)).max() <= F32_ABS_TOL


@pytest.mark.parametrize("d", [1, 5, 32, 96, 128, 200, 256])
def test_f32_head_dims(wf, d):
    q, k, v = (_randn((2, 3, 70, d), 200 + i) for i in range(3))
    out = wf.attention(q.cuda(), k.cuda(), v.cuda()).cpu().numpy()
    assert np.abs(out - _oracle(q, k, v)).max() <= F32_ABS_TOL


def test_f32_hf_strided_views_and_noncausal_and_cross_lengths(wf):
    # HF GPT-2 layout: [B, S, H, D] viewed as [B, H, S, D] without a copy
    base = _randn((2, 77, 3, 12, 64), 300).cuda()
    q, k, v = (base[:, :, i].transpose(1, 2) for i in range(3))
    assert not q.is_contiguous()
    out = wf.attention(q, k, v).cpu().numpy()
    ref = _oracle(q.contiguous().cpu(), k.contiguous().cpu(), v.contiguous().cpu())
    assert np.abs(out - ref).max() <= F32_ABS_TOL
    # non-causal
    out = wf.attention(q, k, v, causal=False).cpu().numpy()
    ref = _oracle(q.contiguous().cpu(), k.contiguous().cpu(), v.contiguous().cpu(), causal=False)
    assert np.abs(out - ref).max() <= F32_ABS_TOL
    # fewer queries than keys (KV-cache step), explicit scale, output into a strided view
    qq = _randn((1, 4, 5, 64), 301)
    kk, vv = (_randn((1, 4, 90, 64), 302 + i) for i in range(2))
    dst = torch.zeros(1, 5, 4, 64, device="cuda")
    wf.attention(qq.cuda(), kk.cuda(), vv.cuda(), scale=0.11, out=dst.transpose(1, 2))
    ref = _oracle(qq, kk, vv, scale=0.11)
    assert np.abs(dst.transpose(1, 2).cpu().numpy() - ref).max() <= F32_ABS_TOL


def test_f32_unaligned_view_takes_the_cuda_core_kernel(wf):
    # q starts 4 bytes into its buffer: not 16-byte aligned, so the TMA-fed tensor-core
    # kernel cannot read it and the call runs on the CUDA-core kernel, at the same contract
    shape = (2, 3, 129, 64)
    n = 2 * 3 * 129 * 64
    base = _randn((n + 1,), 500).cuda()
    q = base[1:].view(shape)
    assert q.data_ptr() % 16 != 0
    k, v = (_randn(shape, 501 + i).cuda() for i in range(2))
    out = wf.attention(q, k, v).cpu().numpy()
    ref = _oracle(q.cpu(), k.cpu(), v.cpu())
    assert np.abs(out - ref).max() <= F32_ABS_TOL
    # the same values from an aligned copy (tensor-core kernel) agree within the contract too
    out_tc = wf.attention(q.clone(), k, v).cpu().numpy()
    assert np.abs(out_tc - ref).max() <= F32_ABS_TOL


def test_f32_gpt2_batched_config3_all_heads(wf):
    # [8, 12, 1024, 64] f32, seed 2: every row of every head against the f64 oracle
    torch.manual_seed(2)
    q, k, v = (torch.randn(8, 12, 1024, 64) for _ in range(3))
    out = wf.attention(q.cuda(), k.cuda(), v.cuda()).cpu().numpy()
    assert np.abs(out - _oracle(q, k, v)).max() <= F32_ABS_TOL


# ---------------------------------------------------------------- bf16 (tcgen05)
@pytest.mark.parametrize("s", [1, 2, 64, 127, 128, 129, 255, 256, 300, 1024, 2048])
def test_bf16_sizes(wf, s):
    q, k, v = (_randn((2, 2, s, 64), 400 + i, torch.bfloat16) for i in range(3))
    out = wf.attention(q.cuda(), k.cuda(), v.cuda()).float().cpu().numpy()
    assert np.isfinite(out).all()
    assert _bf16_rel_err(out, _oracle(q, k, v)) <= BF16_REL_TOL


# The library runs the one-tile kernel when ceil(Sq/256)*B*H is below the SM
# count (148 on B200) and the two-tile kernel otherwise: the small cases above
# take the first, the B*H = 160 cases below the second (one CTA per SM walks
# 160 to 640 work items of 256 query rows, so each CTA runs several).
@pytest.mark.parametrize("s", [1, 100, 129, 256, 300, 1000])
def test_bf16_two_tile_kernel_sizes(wf, s):
    q, k, v = (_randn((2, 80, s, 64), 450 + i, torch.bfloat16) for i in range(3))
    out = wf.attention(q.cuda(), k.cuda(), v.cuda()).float().cpu().numpy()
    assert np.isfinite(out).all()
    flat = (1, 160, s, 64)
    for lo, hi in ((0, 3), (157, 160)):
        ref = _oracle(q, k, v, bh_range=(lo, hi)).reshape(flat)
        assert _bf16_rel_err(out.reshape(flat)[:, lo:hi], ref[:, lo:hi]) <= BF16_REL_TOL


def test_bf16_two_tile_kernel_strided_views(wf):
    # HF layout [B, S, H, D] viewed as [B, H, S, D] for q/k/v and for the output,
    # which the two-tile kernel writes through a TMA tensor map
    base = _randn((2, 300, 3, 80, 64), 470, torch.bfloat16).cuda()
    q, k, v = (base[:, :, i].transpose(1, 2) for i in range(3))
    dst = torch.full((2, 300, 80, 64), float("nan"), dtype=torch.bfloat16, device="cuda")
    wf.attention(q, k, v, out=dst.transpose(1, 2))
    out = dst.transpose(1, 2).float().cpu().numpy().reshape(1, 160, 300, 64)
    qc, kc, vc = (t.contiguous().cpu() for t in (q, k, v))
    ref = _oracle(qc, kc, vc, bh_range=(0, 4)).reshape(1, 160, 300, 64)
    assert np.isfinite(out).all()
    assert _bf16_rel_err(out[:, :4], ref[:, :4]) <= BF16_REL_TOL


def test_bf16_two_tile_kernel_graph_replays(wf):
    # a captured launch of the persistent kernel replayed on new inputs must redo
    # all the work each time
    shape = (1, 160, 300, 64)
    q, k, v = (torch.empty(shape, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    out = torch.empty_like(q)
    wf.attention(q, k, v, out=out)  # first call outside the capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        wf.attention(q, k, v, out=out)
    for rep in range(3):
        src = [_randn(shape, 480 + 3 * rep + i, torch.bfloat16) for i in range(3)]
        for d, h in zip((q, k, v), src):
            d.copy_(h)
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        o = out.float().cpu().numpy()
        assert np.isfinite(o).all(), rep
        ref = _oracle(*src, bh_range=(0, 2))
        assert _bf16_rel_err(o[:, :2], ref[:, :2]) <= BF16_REL_TOL, rep
    del graph


def test_bf16_two_tile_kernel_noncausal_cross_lengths(wf):
    qq = _randn((2, 80, 130, 64), 460, torch.bfloat16)
    kk, vv = (_randn((2, 80, 333, 64), 461 + i, torch.bfloat16) for i in range(2))
    flat_q = (1, 160, 130, 64)
    for causal in (True, False):
        out = wf.attention(qq.cuda(), kk.cuda(), vv.cuda(), causal=causal,
                           scale=0.2).float().cpu().numpy().reshape(flat_q)
        ref = _oracle(qq, kk, vv, causal=causal, scale=0.2, bh_range=(150, 160)).reshape(flat_q)
        assert _bf16_rel_err(out[:, 150:], ref[:, 150:]) <= BF16_REL_TOL


def test_bf16_strided_noncausal_cross_lengths(wf):
    base = _randn((2, 200, 3, 4, 64), 500, torch.bfloat16).cuda()
    q, k, v = (base[:, :, i].transpose(1, 2) for i in range(3))
    out = wf.attention(q, k, v).float().cpu().numpy()
    qc, kc, vc = (t.contiguous().cpu() for t in (q, k, v))
    assert _bf16_rel_err(out, _oracle(qc, kc, vc)) <= BF16_REL_TOL
    out = wf.attention(q, k, v, causal=False).float().cpu().numpy()
    assert _bf16_rel_err(out, _oracle(qc, kc, vc, causal=False)) <= BF16_REL_TOL
    qq = _randn((2, 3, 130, 64), 501, torch.bfloat16)
    kk, vv = (_randn((2, 3, 333, 64), 502 + i, torch.bfloat16) for i in range(2))
    out = wf.attention(qq.cuda(), kk.cuda(), vv.cuda(), scale=0.2).float().cpu().numpy()
    assert _bf16_rel_err(out, _oracle(qq, kk, vv, scale=0.2)) <= BF16_REL_TOL


def test_bf16_config3_against_oracle_and_f32_kernel(wf):
    # [8, 12, 1024, 64], seed 2, bf16 = .bfloat16() of the f32 tensors
    torch.manual_seed(2)
    q, k, v = (torch.randn(8, 12, 1024, 64) for _ in range(3))
    qb, kb, vb = (t.bfloat16() for t in (q, k, v))
    out = wf.attention(qb.cuda(), kb.cuda(), vb.cuda()).float().cpu().numpy()
    # every one of the 96 heads against the f64 oracle (~13 GFLOP, seconds on the host cores)
    ref = _oracle(qb, kb, vb)
    assert _bf16_rel_err(out, ref) <= BF16_REL_TOL
    # size-independent property: the bf16 kernel tracks the f32 kernel on every head
    of32 = wf.attention(qb.float().cuda(), kb.float().cuda(), vb.float().cuda()).cpu().numpy()
    assert _bf16_rel_err(out, of32) <= BF16_REL_TOL


def test_bf16_long_sequence_rows_sampled(wf):
    # one [1, 2, 8192, 64] case (the per-head shape of the long-context workload);
    # the oracle checks the last rows, where all 8192 keys are visible
    q, k, v = (_randn((1, 2, 8192, 64), 600 + i, torch.bfloat16) for i in range(3))
    out = wf.attention(q.cuda(), k.cuda(), v.cuda()).float().cpu().numpy()
    ref = _oracle(q, k, v, row_range=(8192 - 64, 8192))
    o = out[..., -64:, :][None].reshape(1, 2, 64, 64)
    r = ref[..., -64:, :][None].reshape(1, 2, 64, 64)
    assert _bf16_rel_err(o, r) <= BF16_REL_TOL
    ref = _oracle(q, k, v, row_range=(0, 256))
    assert _bf16_rel_err(out[..., :256, :], ref[..., :256, :]) <= BF16_REL_TOL


def test_bf16_two_tile_kernel_grouped_item_order(wf):
    # 18 blocks of 256 rows per head and >= 32 items per SM: the two-tile kernel
    # walks its items in groups of 8 blocks of one head, the last group partial
    b, h, s = 2, 136, 4500
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, v = (torch.randn(b, h, s, 64, generator=g, device="cuda").bfloat16() for _ in range(3))
    out = torch.full_like(q, float("nan"))
    wf.attention(q, k, v, out=out)
    assert torch.isfinite(out.float()).all()
    for bi, hi in ((0, 0), (1, 135), (0, 77), (1, 8)):
        sl = (slice(bi, bi + 1), slice(hi, hi + 1))
        ref = _oracle(q[sl].cpu(), k[sl].cpu(), v[sl].cpu())
        assert _bf16_rel_err(out[sl].float().cpu().numpy(), ref) <= BF16_REL_TOL, (bi, hi)


def test_bf16_gather_writes_every_destination_identically(wf):
    # wfattn_prefill_gather: outputs[0] takes the kernel's TMA stores, outputs[1..] its
    # plain 16-byte stores (the path that writes other GPUs' buffers); here all eight (the
    # most, as on 8 GPUs) are on this GPU, with one strided [B, S, H, D] layout and ragged
    # rows (S = 300)
    b, h, s = 2, 80, 300
    q, k, v = (_randn((b, h, s, 64), 900 + i, torch.bfloat16).cuda() for i in range(3))
    outs = [torch.full((b, s, h, 64), float("nan"), dtype=torch.bfloat16,
                       device="cuda").transpose(1, 2) for _ in range(8)]
    wf.attention_gather(q, k, v, outs)
    ref = wf.attention(q, k, v)
    for o in outs:
        assert torch.equal(o, ref)
    with pytest.raises(ValueError):
        wf.attention_gather(q, k, v, [])
    # the first destination takes TMA stores and must be this GPU's memory: pinned host
    # memory there is rejected on the host before any launch
    from warpforth_b200 import _lib

    host = torch.empty((b, s, h, 64), dtype=torch.bfloat16, pin_memory=True).transpose(1, 2)
    with pytest.raises(_lib.WfattnError, match="outputs\\[0\\]"):
        wf.attention_gather_ptrs(q, k, v, [host.data_ptr(), outs[0].data_ptr()],
                                 outs[0].stride()[:3])


def test_bf16_deterministic_and_output_fully_written(wf):
    q, k, v = (_randn((3, 5, 777, 64), 700 + i, torch.bfloat16).cuda() for i in range(3))
    o1 = torch.full((3, 5, 777, 64), float("nan"), dtype=torch.bfloat16, device="cuda")
    o2 = torch.full_like(o1, float("inf"))
    wf.attention(q, k, v, out=o1)
    wf.attention(q, k, v, out=o2)
    assert torch.isfinite(o1.float()).all()
    assert torch.equal(o1, o2)


def test_no_device_side_timeouts_recorded(wf):
    wf.device_status(clear=True)
