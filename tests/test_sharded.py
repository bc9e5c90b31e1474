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


class _ShmPeerBuffer:
    """Stands in for peer.PeerBuffer on CPU ranks: every rank's buffer is a file in the
    test's folder that all ranks map (shared memory), so a rank's writes land in another
    rank's buffer as the kernel's peer stores do over NVLink.  ``ptrs[r]`` is the address
    of rank r's mapping in this process."""

    def __init__(self, shape, dtype, device, group, root):
        import math

        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        n = math.prod(shape)
        self.maps = [None] * self.world
        self.maps[self.rank] = torch.from_file(f"{root}/peer{self.rank}.bin", shared=True,
                                               size=n, dtype=dtype)
        dist.barrier(group)  # every rank's file exists
        for r in range(self.world):
            if r != self.rank:
                self.maps[r] = torch.from_file(f"{root}/peer{r}.bin", shared=True, size=n,
                                               dtype=dtype)
        self.tensor = self.maps[self.rank].view(shape)
        self.ptrs = [m.data_ptr() for m in self.maps]

    def close(self):
        dist.barrier()


_FAKE_MC_BASE = 1 << 44  # the fake multicast mapping's address of every rank's byte 0


def _race_worker(rank, world, port, result_path, single_slot, transport="peer"):
    """Four steps with different inputs; rank 1 keeps reading each step's output for a while
    (a slow consumer) while rank 0 runs ahead into the next step."""
    import time

    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    from warpforth_b200 import sharded

    root = os.path.dirname(result_path)
    maps = []

    def fake_buffer(shape, dtype, device, group):
        buf = _ShmPeerBuffer(shape, dtype, device, group, root)
        maps.extend(buf.maps)
        return buf

    def fake_gather(q, k, v, out_ptrs, out_strides, *, causal, scale):
        # the "kernel": this rank's output (here q itself) stored into every destination
        for ptr in out_ptrs:
            (m,) = [m for m in maps
                    if m.data_ptr() <= ptr < m.data_ptr() + m.numel() * m.element_size()]
            off = (ptr - m.data_ptr()) // m.element_size()
            torch.as_strided(m, q.shape, (*out_strides, 1), off).copy_(q)

    def fake_mc_buffer(shape, dtype, device, group):
        buf = _ShmPeerBuffer(shape, dtype, device, group, root)
        maps.extend(buf.maps)
        return buf.tensor, buf, _FAKE_MC_BASE

    def fake_multicast(q, k, v, out_mc, out_strides, *, causal, scale):
        # the "kernel": one store through the multicast address lands in every rank's buffer
        for m in maps:
            off = (out_mc - _FAKE_MC_BASE) // m.element_size()
            torch.as_strided(m, q.shape, (*out_strides, 1), off).copy_(q)

    sharded._peer_capable = lambda device, dtype, head_dim: True
    sharded._peer_buffer = fake_buffer
    sharded._launch_gather = fake_gather
    sharded._multicast_capable = lambda device: True
    sharded._multicast_buffer = fake_mc_buffer
    sharded._launch_multicast = fake_multicast
    b, h, s, d = 2, 4, 16, 64
    sp = sharded.ShardedPrefill(b, h, s, d, dtype=torch.bfloat16, device=torch.device("cpu"),
                                transport=transport)
    assert sp.transport == transport
    if single_slot:  # the layout without double buffering: every call writes one slot
        if transport == "peer":
            sp.peer_outs = (sp.peer_outs[0], sp.peer_outs[0])
        else:
            sp.mc_outs = (sp.mc_outs[0], sp.mc_outs[0])
        sp.slots = (sp.slots[0], sp.slots[0])
    report = []
    for step in range(4):
        g = torch.Generator().manual_seed(100 + step)
        q = torch.randn(b, h, s, d, generator=g).bfloat16()
        out = sp(sp.shard(q), sp.shard(q), sp.shard(q))
        seen = out.clone()
        if rank == 1:
            time.sleep(0.5)  # still using this step's output
        report.append(f"{step}:{int(torch.equal(seen, q))}{int(torch.equal(out, seen))}")
    sp.close()
    with open(f"{result_path}.{rank}.status", "w") as f:
        f.write(" ".join(report))
    dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["peer", "multicast"])
@pytest.mark.parametrize("single_slot", [False, True])
def test_peer_output_survives_a_rank_running_ahead(tmp_path, single_slot, transport):
    """The peer and multicast transports' output of call n must stay intact on a slow rank
    while a fast rank runs call n+1 (its stores go to the other slot) until the slow rank's
    next call.  The single-slot layout is run too, to show the test sees the overwrite it
    guards against."""
    port = _free_port()
    path = str(tmp_path / "res")
    mp.start_processes(_race_worker, args=(2, port, path, single_slot, transport), nprocs=2,
                       join=True, start_method="spawn")
    slow = open(f"{path}.1.status").read().split()
    fast = open(f"{path}.0.status").read().split()
    # step:<result right when first read><still intact after the slow read>
    if single_slot:
        # rank 0's next call overwrote the slow rank's output: seen when it first read it
        # or after its slow read, depending on timing
        assert any(r[2:4] != "11" for r in slow[:3]), slow
    else:
        assert [r[2:4] for r in slow] == ["11"] * 4, slow
        assert [r[2] for r in fast] == ["1"] * 4, fast


def test_multicast_transport_needs_cuda_bf16_and_ranks():
    from warpforth_b200 import sharded

    assert sharded._multicast_capable("cpu") is False
    with pytest.raises(ValueError, match="multicast transport needs"):
        sharded.ShardedPrefill(1, 2, 8, 64, dtype=torch.bfloat16, device=torch.device("cpu"),
                               transport="multicast")


def _mc_fallback_worker(rank, world, port, result_path):
    """auto transport where rank 1 cannot set up its multicast buffer: every rank must end up
    on the peer transport."""
    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    from warpforth_b200 import sharded

    root = os.path.dirname(result_path)

    def fake_mc_buffer(shape, dtype, device, group):
        if rank == 1:
            raise RuntimeError("no multicast object for this rank")
        return torch.empty(shape, dtype=dtype), None, _FAKE_MC_BASE

    sharded._peer_capable = lambda device, dtype, head_dim: True
    sharded._multicast_capable = lambda device: True
    sharded._multicast_buffer = fake_mc_buffer
    sharded._peer_buffer = lambda shape, dtype, device, group: _ShmPeerBuffer(
        shape, dtype, device, group, root)
    sp = sharded.ShardedPrefill(2, 4, 16, 64, dtype=torch.bfloat16, device=torch.device("cpu"))
    with open(f"{result_path}.{rank}.status", "w") as f:
        f.write(sp.transport)
    sp.close()
    dist.destroy_process_group()


def test_multicast_setup_failure_on_one_rank_falls_back_to_peer_everywhere(tmp_path):
    path = str(tmp_path / "res")
    mp.start_processes(_mc_fallback_worker, args=(2, _free_port(), path), nprocs=2, join=True,
                       start_method="spawn")
    assert [open(f"{path}.{r}.status").read() for r in range(2)] == ["peer", "peer"]
