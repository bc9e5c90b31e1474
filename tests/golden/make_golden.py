"""Regenerate the golden fixtures in this folder from the reference's own tests.

Run in a checkout that has the reference tree (tetsuo-cpp/warpforth) available:

    python tests/golden/make_golden.py /root/reference

What it does:

1. Imports ``gpu_test/test_kernels.py`` from the reference and runs its three
   attention tests (``test_naive_attention_f64`` :662-712,
   ``test_naive_attention_f64_16x64`` :715-741, ``test_naive_attention_f32``
   :821-875) against a capturing runner.  The runner records the Q/K/V/SEQ_LEN/
   HEAD_DIM parameters each test passes (unpacking the f32-in-i64 packing of
   :805-818 for the f32 test) and answers with the reference's own NumPy
   oracle ``_attention_reference`` (:651-659), so each test's own assertion
   runs and passes.  The captured inputs plus ``_attention_reference``'s output
   are written to ``attention_kats.json``.
2. Builds the seed-0 GPT-2-small attention call (batch 1, 12 heads, seq 64,
   head_dim 64, q/k/v = torch.randn in that order after torch.manual_seed(0))
   and records ``_attention_reference`` per head (f64) and torch's CPU
   ``scaled_dot_product_attention`` (fp32, causal, scale 1/8) in
   ``gpt2_head_call.npz`` together with a checksum of the inputs.

The fixtures are read by tests/ on any machine; this script is the only thing
that reads the reference tree.
"""

from __future__ import annotations

import hashlib
import importlib.util
import json
import struct
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _load_reference_tests(ref_root: Path):
    path = ref_root / "gpu_test" / "test_kernels.py"
    spec = importlib.util.spec_from_file_location("wf_reference_test_kernels", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _unpack_f32(values: list[int], count: int) -> list[float]:
    raw = b"".join(struct.pack("<q", int(v)) for v in values)
    return np.frombuffer(raw, dtype=np.float32)[:count].astype(np.float64).tolist()


def _pack_f32(values: list[float]) -> list[int]:
    b = np.asarray(values, dtype=np.float32).tobytes()
    b += b"\x00" * ((8 - len(b) % 8) % 8)
    return [struct.unpack("<q", b[i:i + 8])[0] for i in range(0, len(b), 8)]


class CapturingRunner:
    """Stands in for the reference KernelRunner: records params, answers with the NumPy oracle."""

    def __init__(self, ref_mod) -> None:
        self.ref = ref_mod
        self.calls: list[dict] = []

    def run(self, forth_source, params=None, grid=(1, 1, 1), block=(1, 1, 1), output_param=0,
            output_count=None):
        s = int(params["SEQ_LEN"])
        d = int(params["HEAD_DIM"])
        packed = "F32@" in forth_source
        arrays = {}
        for name in ("Q", "K", "V"):
            vals = params[name]
            arrays[name] = _unpack_f32(vals, s * d) if packed else [float(x) for x in vals]
        q, k, v = (np.asarray(arrays[n], dtype=np.float64).reshape(s, d) for n in ("Q", "K", "V"))
        expected = self.ref._attention_reference(q, k, v, s)
        self.calls.append({
            "seq_len": s, "head_dim": d, "f32_io": packed,
            "grid": list(grid), "block": list(block), "output_param": output_param,
            "q": arrays["Q"], "k": arrays["K"], "v": arrays["V"], "expected": expected,
        })
        return _pack_f32(expected) if packed else expected


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <root of the reference tree>")
    ref = _load_reference_tests(Path(sys.argv[1]))

    kats = {}
    for test_name, rel in (("test_naive_attention_f64", 1e-6),
                           ("test_naive_attention_f64_16x64", 1e-6),
                           ("test_naive_attention_f32", 1e-5)):
        runner = CapturingRunner(ref)
        getattr(ref, test_name)(runner)  # the reference test's own assertion runs here
        (call,) = runner.calls
        call["rel_tol"] = rel
        kats[test_name] = call
    (HERE / "attention_kats.json").write_text(json.dumps(
        {"source": "gpu_test/test_kernels.py:651-875 (tetsuo-cpp/warpforth)",
         "generator": "tests/golden/make_golden.py", "cases": kats}, indent=1))

    import torch

    torch.manual_seed(0)
    q = torch.randn(1, 12, 64, 64)
    k = torch.randn(1, 12, 64, 64)
    v = torch.randn(1, 12, 64, 64)
    sdpa = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1 / 8)
    ref_out = np.stack([
        np.asarray(ref._attention_reference(q[0, h].double().numpy(), k[0, h].double().numpy(),
                                            v[0, h].double().numpy(), 64)).reshape(64, 64)
        for h in range(12)])[None]
    digest = hashlib.sha256(b"".join(t.numpy().tobytes() for t in (q, k, v))).hexdigest()
    np.savez_compressed(HERE / "gpt2_head_call.npz", reference_f64=ref_out,
                        torch_sdpa_f32=sdpa.numpy(), input_sha256=np.array(digest))
    print("wrote", HERE / "attention_kats.json", HERE / "gpt2_head_call.npz")


if __name__ == "__main__":
    main()
