"""GPT-2 generation with every attention routed through libwfattn.

Mirrors demo/gpt2_generate.py (tetsuo-cpp/warpforth): Hugging Face's
``modeling_gpt2.eager_attention_forward`` is replaced by a function that calls
the WarpForth attention kernel.  The reference loops over heads of batch entry
0 and launches one kernel per head (demo/gpt2_generate.py:35-52); here one
``attention`` call covers every batch entry and head, reads the strided
q/k/v views without copies, and runs on torch's current stream.

Semantics kept from the reference: causal masking only -- ``attention_mask``
(padding) and ``dropout`` are ignored, exactly as the reference ignores them;
``scaling`` is honoured (GPT-2 passes 1/sqrt(head_dim), the reference kernel's
fixed scale).  With a KV cache (``use_cache=True``, which the reference does
not support) the prompt goes through the prefill kernel and every later
single-token step through the split-KV decode kernel (``wfattn_decode_f32``
for the f32 model) over the cached keys and values.

    python -m warpforth_b200.gpt2 --max-tokens 128      # random-init GPT-2 small
"""

from __future__ import annotations

import argparse
import time
from collections.abc import Callable

import torch

from .warpforth import DecodeWorkspace, attention, decode


# library calls made by the patched attention, by kind (read by count_calls)
_calls = {"prefill": 0, "decode": 0}


def make_warpforth_eager_attn() -> Callable:
    """Replacement for transformers' eager_attention_forward (see the module docstring)."""

    workspace = DecodeWorkspace()
    lens_cache: dict = {}

    def warpforth_eager_attn(module, query, key, value, attention_mask=None, scaling=None,
                             dropout=0.0, **kwargs):
        b, _, sq, d = query.shape
        sk = key.shape[2]
        if (sq == 1 and sk > 1 and query.dtype in (torch.float32, torch.bfloat16)
                and d == 64 and key.stride(2) == d and value.stride(2) == d
                and key.stride(3) == 1 and value.stride(3) == 1):
            # one new token against the cached keys: the decode kernel
            _calls["decode"] += 1
            lens = lens_cache.get((b, sk, query.device))
            if lens is None:
                lens = torch.full((b,), sk, dtype=torch.int32, device=query.device)
                lens_cache[(b, sk, query.device)] = lens
            out = decode(query, key, value, lens, scale=scaling, workspace=workspace)
            return out.to(query.dtype).unsqueeze(1), None
        _calls["prefill"] += 1
        out = attention(query, key, value, causal=True, scale=scaling)
        return out.transpose(1, 2), None

    return warpforth_eager_attn


def count_calls(fn: Callable[[], object]) -> dict:
    """Runs fn() and returns how many prefill and decode calls the patched attention made."""
    before = dict(_calls)
    fn()
    return {k: _calls[k] - before[k] for k in _calls}


def patch_gpt2() -> Callable[[], None]:
    """Route GPT-2 attention through libwfattn; returns a function that undoes it."""
    import transformers.models.gpt2.modeling_gpt2 as gpt2_module

    original = gpt2_module.eager_attention_forward
    gpt2_module.eager_attention_forward = make_warpforth_eager_attn()

    def restore() -> None:
        gpt2_module.eager_attention_forward = original

    return restore


def random_gpt2(seed: int = 1, device: str | torch.device = "cuda"):
    """GPT-2 small (12 layers, d_model 768, 12 heads, vocab 50257, ctx 1024), N(0, 0.02) init."""
    from transformers import GPT2Config, GPT2LMHeadModel

    cfg = GPT2Config(n_layer=12, n_embd=768, n_head=12, vocab_size=50257, n_positions=1024,
                     initializer_range=0.02)
    cfg._attn_implementation = "eager"
    torch.manual_seed(seed)
    model = GPT2LMHeadModel(cfg).to(device).float().eval()
    return model


def synthetic_prompt(length: int = 32, seed: int = 1) -> torch.Tensor:
    return torch.randint(0, 50257, (1, length), generator=torch.Generator().manual_seed(seed))


@torch.no_grad()
def generate(model, prompt: torch.Tensor, max_new_tokens: int, use_cache: bool = False):
    ids = prompt.to(next(model.parameters()).device)
    return model.generate(ids, attention_mask=torch.ones_like(ids),
                          max_new_tokens=max_new_tokens, min_new_tokens=max_new_tokens,
                          do_sample=False, use_cache=use_cache, pad_token_id=50256)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--max-tokens", type=int, default=128)
    ap.add_argument("--prompt-len", type=int, default=32)
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--use-cache", action="store_true")
    args = ap.parse_args()
    model = random_gpt2(args.seed)
    prompt = synthetic_prompt(args.prompt_len, args.seed)
    restore = patch_gpt2()
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = generate(model, prompt, args.max_tokens, use_cache=args.use_cache)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
    finally:
        restore()
    print(out[0].tolist())
    print(f"{args.max_tokens / dt:.1f} tokens/s ({out.shape[1]} tokens total)")


if __name__ == "__main__":
    main()
