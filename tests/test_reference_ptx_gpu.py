"""libwfattn against the reference's own compiled kernel (demo/attention.ptx), on the GPU.

The reference's attention kernel exists only compiled (the compiler needs
MLIR 20, absent here), so it is loaded opaquely through the CUDA driver API,
exactly as the reference's binding and runner load it (demo/warpforth.py:26-49,
tools/warpforth-runner/warpforth-runner.cpp:297-321), and launched with the
reference geometry grid = block = (S, 1, 1).  Its output is the parity target:
libwfattn's f32 path must agree with it to 1e-5 absolute, per head, on the
reference's valid domain 2 <= S <= 1024.  The reference's f32 test case also
runs through the runner's PTX path as the reference's harness runs it
(gpu_test/test_kernels.py:821-875).  Skipped when the compiled kernel was not
copied into oracle/_ref (make -C oracle ref).
"""

from __future__ import annotations

import struct
import subprocess

import numpy as np
import pytest

from conftest import ROOT, approx_list
from oracle import ref_ptx

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

F32_ABS_TOL = 1e-5


@pytest.fixture(scope="module")
def kernels():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not ref_ptx.available():
        pytest.skip("the reference's compiled kernel is not in oracle/_ref")
    from warpforth_b200 import warpforth

    return ref_ptx.ReferencePtxKernel(), warpforth


def _per_head_reference(ref, q, k, v):
    """One reference launch per (batch, head), as demo/gpt2_generate.py:42-50 does."""
    b, h, s, d = q.shape
    out = torch.zeros_like(q)
    for bi in range(b):
        for hi in range(h):
            ref(q[bi, hi], k[bi, hi], v[bi, hi], out[bi, hi], s, d)
    return out


def test_matches_compiled_reference_kernel_gpt2_head_call(kernels, gpt2_head_golden):
    ref, wf = kernels
    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 12, 64, 64).cuda() for _ in range(3))
    want = _per_head_reference(ref, q, k, v)
    got = wf.attention(q, k, v)
    one = torch.empty_like(q)
    kern = wf.AttentionKernel()
    for h in range(12):
        kern(q[0, h], k[0, h], v[0, h], one[0, h], 64, 64)
    torch.cuda.synchronize()
    w = want.cpu().numpy()
    assert np.isfinite(w).all()
    assert np.abs(w - gpt2_head_golden["reference_f64"]).max() <= F32_ABS_TOL
    for out in (got, one):
        assert np.abs(out.cpu().numpy() - w).max() <= F32_ABS_TOL


@pytest.mark.parametrize("s", [2, 3, 17, 63, 64, 65, 129, 500, 1024])
@pytest.mark.parametrize("d", [4, 64])
def test_matches_compiled_reference_kernel_sizes(kernels, s, d):
    ref, wf = kernels
    g = torch.Generator().manual_seed(1000 + s + d)
    q, k, v = (torch.randn(1, 1, s, d, generator=g).cuda() for _ in range(3))
    want = _per_head_reference(ref, q, k, v)
    got = wf.attention(q, k, v)
    assert np.abs(got.cpu().numpy() - want.cpu().numpy()).max() <= F32_ABS_TOL


def test_matches_compiled_reference_kernel_config3_every_head(kernels):
    # [8, 12, 1024, 64] f32, seed 2: 96 reference launches against one batched call
    ref, wf = kernels
    torch.manual_seed(2)
    q, k, v = (torch.randn(8, 12, 1024, 64).cuda() for _ in range(3))
    want = _per_head_reference(ref, q, k, v)
    got = wf.attention(q, k, v)
    assert np.abs(got.cpu().numpy() - want.cpu().numpy()).max() <= F32_ABS_TOL


def test_reference_kernel_domain_is_guarded(kernels):
    ref, _ = kernels
    t = torch.zeros(2048 * 64, device="cuda")
    for s in (1, 1025):
        with pytest.raises(ref_ptx.ReferencePtxError, match="SEQ_LEN"):
            ref(t, t, t, t, s, 64)


def _pack(values) -> str:
    b = np.asarray(values, dtype=np.float32).tobytes()
    b += b"\x00" * ((8 - len(b) % 8) % 8)
    return ",".join(str(struct.unpack("<q", b[i:i + 8])[0]) for i in range(0, len(b), 8))


def _unpack(csv: str, count: int) -> list[float]:
    raw = b"".join(struct.pack("<q", int(x)) for x in csv.strip().split(","))
    return np.frombuffer(raw, dtype=np.float32)[:count].tolist()


def test_reference_f32_case_through_runner_both_paths(kernels, kats):
    """The reference's f32 attention test, command line as its harness builds it, run by
    wfattn-runner on the compiled reference kernel (--impl ptx) and on libwfattn."""
    runner = ROOT / "warpforth_b200" / "lib" / "wfattn-runner"
    if not runner.exists():
        pytest.skip("wfattn-runner not built")
    c = kats["test_naive_attention_f32"]
    s, d = c["seq_len"], c["head_dim"]
    n_i64 = (s * d + 1) // 2
    args = ["--kernel", "attention",
            "--param", f"i64[]:{_pack(c['q'])}", "--param", f"i64[]:{_pack(c['k'])}",
            "--param", f"i64[]:{_pack(c['v'])}", "--param", "i64[]:" + ",".join(["0"] * n_i64),
            "--param", f"i64:{s}", "--param", f"i64:{d}", "--grid", f"{s},1,1",
            "--block", f"{s},1,1", "--output-param", "3", "--output-count", str(n_i64)]
    outs = {}
    for impl in ("ptx", "wfattn"):
        res = subprocess.run([str(runner), str(ref_ptx.PTX_PATH), *args, "--impl", impl],
                             capture_output=True, text=True, timeout=120)
        assert res.returncode == 0, res.stderr
        outs[impl] = _unpack(res.stdout, s * d)
        assert outs[impl] == approx_list(c["expected"], rel=c["rel_tol"])
    assert np.abs(np.array(outs["ptx"]) - np.array(outs["wfattn"])).max() <= F32_ABS_TOL


def test_gpt2_tokens_through_compiled_reference_kernel(kernels):
    """Greedy GPT-2 (random init, seed 1) through the reference's per-head demo patch on its
    compiled kernel gives the same token ids as through libwfattn's batched patch."""
    ref, _ = kernels
    import transformers.models.gpt2.modeling_gpt2 as gpt2_module

    from warpforth_b200 import gpt2

    model = gpt2.random_gpt2(seed=1, device="cuda")
    prompt = gpt2.synthetic_prompt(32, seed=1)
    original = gpt2_module.eager_attention_forward
    try:
        gpt2_module.eager_attention_forward = ref_ptx.make_reference_eager_attn(ref)
        want = gpt2.generate(model, prompt, 24).cpu()
    finally:
        gpt2_module.eager_attention_forward = original
    restore = gpt2.patch_gpt2()
    try:
        got = gpt2.generate(model, prompt, 24).cpu()
    finally:
        restore()
    assert torch.equal(got, want)
