"""Head-sharded multi-GPU causal prefill with an all-gather of the output.

Every (batch, head) pair of attention is independent, so G ranks (one process
per GPU) split the heads evenly and compute them with no exchange; the only
exchange is the all-gather of O.  Three transports:

* ``multicast`` (bf16 on GPUs with NVLS, the default there): every rank holds
  two full [B, H, S, D] output slots in one symmetric-memory buffer
  (``torch.distributed._symmetric_memory``) that all ranks have bound to one
  NVLink multicast object.  The attention kernel writes each finished output
  tile of its heads once through the multicast address
  (``wfattn_prefill_multicast``, ``multimem.st``) and the NVLink switch
  delivers it to every rank's buffer: a rank's NVLink egress is its own share
  of O, not (G - 1) copies of it.  Slots and the closing barrier as for peer.
* ``peer`` (bf16 on GPUs without NVLS): every rank holds two full
  [B, H, S, D] output slots in one ``peer.PeerBuffer`` mapped on all ranks
  (CUDA IPC).  The attention kernel stores each finished output tile of its
  heads into every rank's buffer over NVLink (``wfattn_prefill_gather``), so
  the gather rides along tile by tile with the compute; one cross-rank barrier
  ends the step.  Rank r owns heads [r*H/G, (r+1)*H/G).  Calls alternate
  between the two slots: a rank that starts call n+1 early writes the other
  slot, and it cannot start call n+2 (which reuses call n's slot) before every
  rank has reached the barrier of call n+1, i.e. before every rank has queued
  or finished whatever it does with call n's output.
* ``nccl`` (any dtype or device, and the fallback): the heads are cut into C
  chunks of H/C heads, each chunk split evenly over the ranks: rank r owns
  heads [c*H/C + r*h, c*H/C + (r+1)*h) of chunk c, with h = H/(C*G).  A rank
  computes its part of chunk c, then starts the all-gather of chunk c
  (asynchronously, on the collective's own stream) while it computes chunk
  c+1.  Each rank writes its heads into its slot of a head-major buffer
  [C, G, h, B, S, D]; the gathers run in place, and the buffer is exactly a
  strided [B, H, S, D] view (no copy):

      gathered.view(H, B, S, D).permute(1, 0, 2, 3)  ->  [B, H, S, D]

The NCCL transport goes through ``torch.distributed`` (gloo on CPU for the
tests); its per-rank compute is injectable so that the shard/gather logic can
be tested on CPU ranks against the oracle.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch
import torch.distributed as dist


def head_range(heads: int, world: int, rank: int) -> tuple[int, int]:
    """Heads owned by `rank` of `world` with one chunk (an even split; heads % world == 0)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if heads % world:
        raise ValueError(f"{heads} heads cannot be split evenly over {world} ranks")
    per = heads // world
    return rank * per, (rank + 1) * per


def default_chunks(heads: int, world: int) -> int:
    """Chunks for overlapping the gather with compute: 1 on one rank, else the largest of
    3 and 2 that divides the heads per rank (1 if neither does)."""
    if world == 1:
        return 1
    per = heads // world
    return next((c for c in (3, 2) if per % c == 0), 1)


ComputeFn = Callable[..., torch.Tensor]


def _peer_capable(device, dtype, head_dim) -> bool:
    """Whether the kernel-side peer gather can run for this device, dtype and head size."""
    return torch.device(device).type == "cuda" and dtype == torch.bfloat16 and head_dim == 64


class MulticastSetupError(RuntimeError):
    """Some rank has no usable multicast mapping (raised on every rank)."""


def _multicast_capable(device) -> bool:
    """Whether torch's symmetric memory offers an NVLS multicast mapping on this device."""
    device = torch.device(device)
    if device.type != "cuda":
        return False
    try:
        from torch.distributed._symmetric_memory import DeviceType, _SymmetricMemory

        return bool(_SymmetricMemory.has_multicast_support(DeviceType.CUDA, device.index or 0))
    except (ImportError, AttributeError, RuntimeError):
        return False


def _multicast_buffer(shape, dtype, device, group):
    """(this rank's buffer, a handle that keeps the mapping alive, the multicast address of
    the buffer's first byte or 0).  Collective.  The kernel addresses the output as
    multicast base + byte offset, so the address is given only when the tensor starts
    its allocation: then the multicast base and this rank's buffer base describe the
    same bytes."""
    import torch.distributed._symmetric_memory as symm_mem

    buf = symm_mem.empty(shape, dtype=dtype, device=device)
    hdl = symm_mem.rendezvous(buf, group if group is not None else dist.group.WORLD)
    mc = int(hdl.multicast_ptr) if hdl.multicast_ptr else 0
    rank = dist.get_rank(group)
    if mc % 16 or int(hdl.offset) != 0 or buf.data_ptr() != int(hdl.buffer_ptrs[rank]):
        mc = 0
    return buf, hdl, mc


def _launch_multicast(q, k, v, out_mc, out_strides, *, causal, scale):
    from .warpforth import attention_multicast_ptr

    attention_multicast_ptr(q, k, v, out_mc, out_strides, causal=causal, scale=scale)


def _peer_buffer(shape, dtype, device, group):
    from .peer import PeerBuffer

    return PeerBuffer(shape, dtype, device, group)


def _launch_gather(q, k, v, out_ptrs, out_strides, *, causal, scale):
    from .warpforth import attention_gather_ptrs

    attention_gather_ptrs(q, k, v, out_ptrs, out_strides, causal=causal, scale=scale)


def _default_compute(q, k, v, *, causal, scale, out):
    from .warpforth import attention

    return attention(q, k, v, causal=causal, scale=scale, out=out)


class ShardedPrefill:
    """Runs this rank's share of a [B, H, S, D] attention and all-gathers O.

    The output buffers (two slots of [B, H, S, D] for the multicast and peer transports,
    ``gathered`` = [C, G, h, B, S, D] for NCCL) are allocated once and reused.
    ``__call__`` takes this rank's q/k/v as per-chunk lists of [B, h, S, D]
    views (from ``shard`` of the full tensors or ``split_local`` of a
    rank-local tensor; one chunk with multicast or peer) and returns the full
    [B, H, S, D] output.  ``transport`` is "auto" (multicast, else peer, where
    possible), "multicast", "peer" or "nccl".

    Lifetime of the returned tensor: it holds this call's output until the
    call after next (multicast and peer: the two slots alternate; NCCL: the
    gather buffer is reused by the next call).  Whatever reads it must be
    queued on the current stream, or finished on the host, before this rank's
    next call; other ranks cannot overwrite it before then.
    """

    def __init__(self, batch: int, heads: int, seq: int, head_dim: int, *,
                 dtype: torch.dtype, device: torch.device, group=None,
                 compute: ComputeFn | None = None, chunks: int | None = None,
                 transport: str = "auto") -> None:
        if transport not in ("auto", "multicast", "peer", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        head_range(heads, self.world, self.rank)  # validates the even split
        self.local_heads = heads // self.world
        self.B, self.H, self.S, self.D = batch, heads, seq, head_dim
        self.transport = "nccl"
        self.peer = None
        self.mc_buf = self.mc_handle = None
        peer_ok = (self.world > 1 and _peer_capable(device, dtype, head_dim)
                   and compute is None and chunks in (None, 1))
        if transport in ("peer", "multicast") and not peer_ok:
            raise ValueError(f"the {transport} transport needs bf16, head_dim 64, CUDA and "
                             ">1 rank")
        if transport in ("auto", "multicast") and peer_ok:
            try:  # collective; every rank agrees before and after the rendezvous
                self._setup_multicast(dtype, device)
                self.transport = "multicast"
            except MulticastSetupError:
                if transport == "multicast":
                    raise
        if self.transport == "nccl" and transport in ("auto", "peer") and peer_ok:
            from .peer import PeerSetupError

            try:  # collective; on failure every rank raises, so all of them fall back
                self._setup_peer(dtype, device)
                self.transport = "peer"
            except PeerSetupError:
                if transport == "peer":
                    raise
        if self.transport in ("multicast", "peer"):
            self.chunks, self.ch = 1, self.local_heads
            return
        self.chunks = chunks or default_chunks(heads, self.world)
        if self.local_heads % self.chunks:
            raise ValueError(f"{self.local_heads} heads per rank cannot form {self.chunks} chunks")
        self.ch = self.local_heads // self.chunks
        self.gathered = torch.empty((self.chunks, self.world, self.ch, batch, seq, head_dim),
                                    dtype=dtype, device=device)
        self.compute = compute or _default_compute

    def _agree(self, ok: bool, device) -> bool:
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        return bool(int(flag.item()))

    def _setup_multicast(self, dtype, device) -> None:
        if not self._agree(_multicast_capable(device), device):
            raise MulticastSetupError("no NVLS multicast support on some rank")
        try:
            buf, hdl, mc = _multicast_buffer((2, self.B, self.H, self.S, self.D), dtype, device,
                                             self.group)
        except RuntimeError:  # this rank could not allocate or map; all ranks learn it next
            buf = hdl = None
            mc = 0
        if not self._agree(mc != 0, device):
            raise MulticastSetupError("no multicast address at the start of the output buffer")
        self.mc_buf, self.mc_handle = buf, hdl
        self.slots = (buf[0], buf[1])
        esz = buf.element_size()
        head_off = self.rank * self.local_heads * buf.stride(2) * esz
        slot_bytes = buf.stride(0) * esz
        self.mc_outs = tuple(mc + s * slot_bytes + head_off for s in (0, 1))
        self.out_strides = buf.stride()[1:4]
        self.calls = 0
        self._sync = torch.zeros(1, dtype=torch.int32, device=device)

    def _setup_peer(self, dtype, device) -> None:
        # two output slots [2, B, H, S, D] in one buffer per rank, mapped on every rank
        self.peer = _peer_buffer((2, self.B, self.H, self.S, self.D), dtype, device, self.group)
        buf = self.peer.tensor
        self.slots = (buf[0], buf[1])
        esz = buf.element_size()
        # this rank's heads inside every rank's output slot, as mapped on this GPU; its
        # own buffer first (the kernel's TMA tensor stores go to the first destination
        # only, the other GPUs' buffers get bulk copies of the same output slabs)
        head_off = self.rank * self.local_heads * buf.stride(2) * esz
        slot_bytes = buf.stride(0) * esz
        order = [self.rank] + [r for r in range(self.world) if r != self.rank]
        self.peer_outs = tuple([self.peer.ptrs[r] + s * slot_bytes + head_off for r in order]
                               for s in (0, 1))
        self.out_strides = buf.stride()[1:4]
        self.calls = 0  # peer calls so far; call n writes slot n % 2
        self._sync = torch.zeros(1, dtype=torch.int32, device=device)

    def close(self) -> None:
        """Collective with the peer transport (every rank calls it): releases the mapped
        output buffers.  Without it they live until the process exits."""
        if self.transport == "peer" and self.peer is not None:
            self.slots = None
            self.peer.close()
            self.peer = None
        if self.transport == "multicast" and self.mc_buf is not None:
            # no rank may still write through the multicast mapping when it goes
            if self.mc_buf.device.type == "cuda":
                torch.cuda.synchronize(self.mc_buf.device)
            dist.all_reduce(self._sync, group=self.group)
            self.slots = None
            self.mc_handle = self.mc_buf = None

    def chunk_heads(self, c: int) -> tuple[int, int]:
        """Global head range of this rank's part of chunk c."""
        lo = c * (self.H // self.chunks) + self.rank * self.ch
        return lo, lo + self.ch

    def shard(self, t: torch.Tensor) -> list[torch.Tensor]:
        """This rank's per-chunk head slices of a full [B, H, S, D] tensor (views)."""
        return [t[:, lo:hi] for lo, hi in (self.chunk_heads(c) for c in range(self.chunks))]

    def split_local(self, t: torch.Tensor) -> list[torch.Tensor]:
        """Per-chunk views of a rank-local [B, H/G, S, D] tensor holding this rank's heads in
        chunk order (chunk c = local heads [c*h, (c+1)*h))."""
        return [t[:, c * self.ch:(c + 1) * self.ch] for c in range(self.chunks)]

    def output_view(self) -> torch.Tensor:
        """The full [B, H, S, D] output of the last call."""
        if self.transport in ("multicast", "peer"):
            return self.slots[(self.calls - 1) & 1]
        return self.gathered.view(self.H, self.B, self.S, self.D).permute(1, 0, 2, 3)

    def _compute_chunk(self, c, q, k, v, causal, scale):
        # this rank's [h, B, S, D] slot seen as [B, h, S, D]
        self.compute(q, k, v, causal=causal, scale=scale,
                     out=self.gathered[c, self.rank].permute(1, 0, 2, 3))

    def compute_local(self, qs: Sequence[torch.Tensor], ks: Sequence[torch.Tensor],
                      vs: Sequence[torch.Tensor], *, causal: bool = True,
                      scale: float | None = None) -> None:
        """This rank's heads only, without the final synchronisation (multicast and peer: the
        kernel still stores into every rank's buffer, into the slot the next call
        writes)."""
        if self.transport == "multicast":
            _launch_multicast(qs[0], ks[0], vs[0], self.mc_outs[self.calls & 1],
                              self.out_strides, causal=causal, scale=scale)
            return
        if self.transport == "peer":
            _launch_gather(qs[0], ks[0], vs[0], self.peer_outs[self.calls & 1],
                           self.out_strides, causal=causal, scale=scale)
            return
        for c in range(self.chunks):
            self._compute_chunk(c, qs[c], ks[c], vs[c], causal, scale)

    def __call__(self, qs: Sequence[torch.Tensor], ks: Sequence[torch.Tensor],
                 vs: Sequence[torch.Tensor], *, causal: bool = True,
                 scale: float | None = None) -> torch.Tensor:
        if self.transport in ("multicast", "peer"):
            self.compute_local(qs, ks, vs, causal=causal, scale=scale)
            self.calls += 1
            # A one-element NCCL all-reduce as the cross-rank barrier: once it is
            # done on this rank, every rank's attention kernel (queued before its
            # all-reduce) has completed its stores into this rank's buffer.  It is
            # bounded by the process group's timeout.  It also keeps every rank
            # from starting the call after next -- the next writer of this
            # call's slot -- before this rank has queued the next call.
            dist.all_reduce(self._sync, group=self.group)
            return self.output_view()
        works = []
        for c in range(self.chunks):
            self._compute_chunk(c, qs[c], ks[c], vs[c], causal, scale)
            if self.world > 1:
                works.append(dist.all_gather_into_tensor(
                    self.gathered[c].view(-1), self.gathered[c, self.rank].reshape(-1),
                    group=self.group, async_op=True))
        for w in works:
            w.wait()
        return self.output_view()
