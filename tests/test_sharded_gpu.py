"""Head-sharded prefill on 2 GPUs: every transport against one-GPU results.

multicast: every rank's kernel writes its heads once through an NVLS multicast
address of a symmetric-memory buffer (wfattn_prefill_multicast), where the box
offers multicast; peer: every rank's kernel stores its heads into every rank's
output buffer (CUDA IPC mappings, wfattn_peer_*) over NVLink
(wfattn_prefill_gather).  Both gathered outputs must be bit-identical to the
same kernel run for all heads on one GPU.  No rank leaves early: both end
together after closing the transports.  nccl: chunked all-gathers of per-rank outputs; within the bf16
tolerance of that result.  Three steps with different inputs, and rank 1 reads
each step's output only after a ~25 ms device delay, while rank 0 runs ahead:
its next step must not overwrite what rank 1 has yet to read.  Skipped on boxes
with fewer than two GPUs.
"""

from __future__ import annotations

import socket
import sys
from datetime import timedelta

import numpy as np
import pytest

from conftest import ROOT

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, path):
    sys.path.insert(0, str(ROOT))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    from warpforth_b200 import warpforth as wf
    from warpforth_b200.sharded import ShardedPrefill, _multicast_capable

    b, h, s, d = 2, 16, 640, 64
    steps = []
    for step in range(3):  # different inputs every step
        g = torch.Generator().manual_seed(7 + step)
        q, k, v = (torch.randn(b, h, s, d, generator=g).bfloat16().to(dev) for _ in range(3))
        ref = torch.empty_like(q)
        wf.attention_gather(q, k, v, [ref])  # the two-tile kernel for every head, one GPU
        steps.append((q, k, v, ref))
    torch.cuda.synchronize()
    res = {}
    mc_ok = _multicast_capable(dev)
    for transport in (("multicast",) if mc_ok else ()) + ("peer", "nccl"):
        sp = ShardedPrefill(b, h, s, d, dtype=torch.bfloat16, device=dev, transport=transport)
        exact, rel = True, 0.0
        for q, k, v, ref in steps:
            out = sp(sp.shard(q), sp.shard(k), sp.shard(v))
            if rank == 1:
                # a slow consumer: its copy of this step's output runs ~25 ms later on the
                # GPU, while rank 0 is already in the next step
                torch.cuda._sleep(50_000_000)
            seen = out.clone()
            exact &= bool(torch.equal(seen, ref))
            o = seen.float()
            rel = max(rel, float((o - ref.float()).abs().max() / ref.float().abs().max()))
        torch.cuda.synchronize()
        res[transport] = (sp.transport, exact, rel)
        sp.close()
    mc = res.get("multicast", ("none", True, 0.0))
    np.save(f"{path}.{rank}.npy", np.array([res["peer"][1], res["nccl"][2],
                                             res["peer"][0] == "peer", mc_ok,
                                             mc[0] == "multicast", mc[1]], dtype=np.float64))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_multicast_peer_and_nccl_transports(tmp_path):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = str(tmp_path / "res")
    mp.start_processes(_worker, args=(2, _free_port(), path), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        peer_exact, nccl_rel, used_peer, mc_ok, used_mc, mc_exact = np.load(f"{path}.{r}.npy")
        assert used_peer == 1.0
        assert peer_exact == 1.0
        assert nccl_rel <= 2e-2
        if mc_ok:  # the box offers NVLS multicast: the multicast transport must run, exactly
            assert used_mc == 1.0
            assert mc_exact == 1.0
