"""warpforth_b200 -- B200 (sm_100a) replacement for WarpForth's attention hot path.

The kernels and the C ABI live in libwfattn (``csrc/``, ``include/wfattn.h``);
this package holds the Python side of the drop-in boundary:

* ``warpforth.AttentionKernel`` -- the reference's demo/warpforth.py interface;
* ``warpforth.attention`` / ``warpforth.decode`` -- batched prefill and decode;
* ``gpt2`` -- the GPT-2 attention patch of demo/gpt2_generate.py, batched;
* ``sharded`` -- head-sharded multi-GPU prefill; the kernel stores O into every rank's
  buffer (``peer``: CUDA IPC mappings over NVLink), or NCCL all-gathers it.
"""

from __future__ import annotations

__all__ = ["AttentionKernel", "attention", "attention_gather",
           "attention_gather_ptrs", "decode", "DecodeWorkspace"]


def __getattr__(name):  # lazy: importing the package does not import torch
    if name in __all__:
        from . import warpforth

        return getattr(warpforth, name)
    raise AttributeError(name)
