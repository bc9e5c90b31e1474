"""Head-sharded prefill with an all-gather of O, on CPU ranks over gloo.

Each rank computes only its heads (here with the CPU oracle standing in for
the GPU kernel) into its slot of the head-major gather buffer; after the
in-place all-gather every rank must hold the full [B, H, S, D] output,
identical to a single-process computation.  Also covers the failure paths on
the host: a rank that raises before the collective makes the others' gather
fail with the group timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from conftest import ROOT  # noqa: E402


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_compute(q, k, v, *, causal, scale, out):
    import oracle

    res = oracle.attention(q.contiguous().numpy(), k.contiguous().numpy(),
                           v.contiguous().numpy(), causal=causal, scale=scale)
    out.copy_(torch.from_numpy(res))
    return out


def _inputs():
    g = torch.Generator().manual_seed(4)
    return tuple(torch.randn(2, 6, 40, 16, generator=g) for _ in range(3))


def _worker(rank, world, port, result_path, mode):
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=10))
    from warpforth_b200.sharded import ShardedPrefill

    q, k, v = _inputs()
    sp = ShardedPrefill(2, 6, 40, 16, dtype=torch.float32, device=torch.device("cpu"),
                        compute=_oracle_compute, chunks=1 if mode == "chunks1" else None)
    status = "ok"
    try:
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before the collective")
        if mode == "local":
            # a rank-local [B, H/G, S, D] tensor of this rank's heads in chunk order
            qs, ks, vs = (sp.split_local(torch.cat(sp.shard(t), dim=1)) for t in (q, k, v))
            out = sp(qs, ks, vs)
        else:
            out = sp(sp.shard(q), sp.shard(k), sp.shard(v))
        np.save(f"{result_path}.{rank}.npy", out.contiguous().numpy())
    except RuntimeError as e:
        status = f"error: {e}"
    with open(f"{result_path}.{rank}.status", "w") as f:
        f.write(status)
    if mode != "fail":
        dist.destroy_process_group()


def _spawn(world, tmp_path, mode):
    port = _free_port()
    path = str(tmp_path / "res")
    mp.start_processes(_worker, args=(world, port, path, mode), nprocs=world, join=True,
                       start_method="spawn")
    return path


def test_head_range_even_split():
    from warpforth_b200.sharded import head_range

    assert [head_range(48, 8, r) for r in range(8)] == [(6 * r, 6 * r + 6) for r in range(8)]
    assert head_range(12, 1, 0) == (0, 12)
    with pytest.raises(ValueError):
        head_range(48, 5, 0)
    with pytest.raises(ValueError):
        head_range(48, 2, 2)


def test_sharded_gather_matches_single_process(tmp_path):
    import oracle

    path = _spawn(2, tmp_path, "ok")
    q, k, v = _inputs()
    ref = oracle.attention(q.numpy(), k.numpy(), v.numpy())
    for r in range(2):
        assert open(f"{path}.{r}.status").read() == "ok"
        out = np.load(f"{path}.{r}.npy")
        assert out.shape == (2, 6, 40, 16)
        assert np.array_equal(out, ref)


@pytest.mark.parametrize("mode", ["chunks1", "local"])
def test_sharded_gather_one_chunk_and_rank_local_inputs(tmp_path, mode):
    import oracle

    path = _spawn(2, tmp_path, mode)
    q, k, v = _inputs()
    ref = oracle.attention(q.numpy(), k.numpy(), v.numpy())
    for r in range(2):
        assert open(f"{path}.{r}.status").read() == "ok"
        assert np.array_equal(np.load(f"{path}.{r}.npy"), ref)


def test_chunk_head_assignment_covers_every_head_once():
    from warpforth_b200 import sharded

    for heads, world in ((48, 8), (48, 4), (48, 2), (12, 3), (6, 2)):
        chunks = sharded.default_chunks(heads, world)
        seen = []
        for c in range(chunks):
            for rank in range(world):
                sp = object.__new__(sharded.ShardedPrefill)  # rank's view, no process group
                sp.H, sp.chunks, sp.rank, sp.ch = heads, chunks, rank, heads // world // chunks
                lo, hi = sp.chunk_heads(c)
                seen += list(range(lo, hi))
        # gathered[c, rank, i] holds head chunk_heads(c)[0] + i: head-major order
        assert seen == list(range(heads)), (heads, world, chunks)


def test_single_rank_output_view_is_full_tensor():
    from warpforth_b200.sharded import ShardedPrefill

    q, k, v = _inputs()
    sp = ShardedPrefill(2, 6, 40, 16, dtype=torch.float32, device=torch.device("cpu"),
                        compute=_oracle_compute)
    out = sp(sp.shard(q), sp.shard(k), sp.shard(v))
    import oracle

    assert np.array_equal(out.contiguous().numpy(), oracle.attention(q.numpy(), k.numpy(),
                                                                     v.numpy()))
    assert out.data_ptr() == sp.gathered.data_ptr()  # a view, not a copy


def test_failed_rank_surfaces_as_collective_error(tmp_path):
    path = _spawn(2, tmp_path, "fail")
    assert open(f"{path}.1.status").read().startswith("error: rank 1 fails")
    st0 = open(f"{path}.0.status").read()
    assert st0.startswith("error:"), st0


class _FakePeerLib:
    """Stands in for libwfattn's peer-buffer calls on a CPU rank: allocation and mapping
    succeed or fail as told, and every call is recorded."""

    def __init__(self, alloc_ok: bool, open_ok: bool) -> None:
        self.alloc_ok, self.open_ok, self.calls = alloc_ok, open_ok, []

    def wfattn_peer_alloc(self, nbytes, device, ptr, handle):
        self.calls.append("alloc")
        if not self.alloc_ok:
            return 3
        ptr._obj.value = 1 << 20
        handle._obj.bytes[0] = 7
        return 0

    def wfattn_peer_open(self, handle, device, ptr):
        self.calls.append("open")
        if not self.open_ok:
            return 3
        ptr._obj.value = 2 << 20
        return 0

    def wfattn_peer_close(self, ptr, device):
        self.calls.append("close")
        return 0

    def wfattn_peer_free(self, ptr, device):
        self.calls.append("free")
        return 0


def _peer_worker(rank, world, port, result_path, case):
    import types

    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=10))
    from warpforth_b200 import _lib, peer

    alloc_ok = not (case == "alloc" and rank == 0)
    open_ok = not (case == "open" and rank == 1)
    fake = _FakePeerLib(alloc_ok, open_ok)

    def check(status):
        if status:
            raise _lib.WfattnError(status, "fake failure")

    def load():
        if case == "load" and rank == 0:
            raise _lib.WfattnError(_lib.CUDA_ERROR, "library missing")
        return fake

    peer._lib = types.SimpleNamespace(load=load, check=check, PeerHandle=_lib.PeerHandle,
                                      WfattnError=_lib.WfattnError)
    try:
        peer.PeerBuffer((2, 4, 8, 64), torch.bfloat16, torch.device("cuda", rank))
        status = "no error"
    except peer.PeerSetupError as e:
        status = f"PeerSetupError: {e}"
    with open(f"{result_path}.{rank}.status", "w") as f:
        f.write(status + "\n" + ",".join(fake.calls))
    dist.destroy_process_group()


@pytest.mark.parametrize("case", ["alloc", "open", "load"])
def test_peer_buffer_setup_failure_is_raised_on_every_rank(tmp_path, case):
    """One rank's failed library load or allocation (rank 0) or mapping (rank 1) makes every
    rank raise PeerSetupError after releasing what it set up, so all ranks can fall back
    together."""
    port = _free_port()
    path = str(tmp_path / "res")
    mp.start_processes(_peer_worker, args=(2, port, path, case), nprocs=2, join=True,
                       start_method="spawn")
    out = {r: open(f"{path}.{r}.status").read().split("\n") for r in range(2)}
    for r in range(2):
        assert out[r][0].startswith("PeerSetupError: rank "), out[r]
    if case == "load":
        assert out[0][1] == ""  # never reached the library
        assert out[1][1] == "alloc,free"
        assert "rank 0: " in out[1][0] and "library missing" in out[1][0]
    elif case == "alloc":
        assert out[0][1] == "alloc"  # nothing to release
        assert out[1][1] == "alloc,free"  # never maps, frees its own buffer
        assert "rank 0" in out[1][0]
    else:
        assert out[0][1] == "alloc,open,close,free"  # unmaps rank 1's buffer, frees its own
        assert out[1][1] == "alloc,open,free"  # its mapping failed: only frees its own
        assert "rank 1" in out[0][0]
