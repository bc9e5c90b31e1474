"""Head-sharded multi-GPU causal prefill with an all-gather of the output.

Every (batch, head) pair of attention is independent, so G ranks (one process
per GPU) split the heads evenly and compute them with no exchange; the only
collective is the all-gather of O.  To hide that gather behind compute, the
heads are cut into C chunks of H/C heads, each chunk split evenly over the
ranks: rank r owns heads [c*H/C + r*h, c*H/C + (r+1)*h) of chunk c, with
h = H/(C*G).  A rank computes its part of chunk c, then starts the all-gather
of chunk c (asynchronously, on the collective's own stream) while it computes
chunk c+1.

Each rank writes its heads into its slot of a head-major buffer
[C, G, h, B, S, D]; the gathers run in place, and the buffer is exactly a
strided [B, H, S, D] view (no copy):

    gathered.view(H, B, S, D).permute(1, 0, 2, 3)  ->  [B, H, S, D]

The collective goes through ``torch.distributed`` (NCCL over NVLink on GPUs,
gloo on CPU for the tests).  The per-rank compute is injectable so that the
shard/gather logic can be tested on CPU ranks against the oracle.
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


def _default_compute(q, k, v, *, causal, scale, out):
    from .warpforth import attention

    return attention(q, k, v, causal=causal, scale=scale, out=out)


class ShardedPrefill:
    """Runs this rank's share of a [B, H, S, D] attention and all-gathers O.

    ``gathered`` ([C, G, h, B, S, D]) is allocated once and reused.  ``__call__``
    takes this rank's q/k/v as per-chunk lists of [B, h, S, D] views (from
    ``shard`` of the full tensors or ``split_local`` of a rank-local tensor)
    and returns the full output as a [B, H, S, D] view of ``gathered``.
    """

    def __init__(self, batch: int, heads: int, seq: int, head_dim: int, *,
                 dtype: torch.dtype, device: torch.device, group=None,
                 compute: ComputeFn | None = None, chunks: int | None = None) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        head_range(heads, self.world, self.rank)  # validates the even split
        self.local_heads = heads // self.world
        self.chunks = chunks or default_chunks(heads, self.world)
        if self.local_heads % self.chunks:
            raise ValueError(f"{self.local_heads} heads per rank cannot form {self.chunks} chunks")
        self.ch = self.local_heads // self.chunks
        self.B, self.H, self.S, self.D = batch, heads, seq, head_dim
        self.gathered = torch.empty((self.chunks, self.world, self.ch, batch, seq, head_dim),
                                    dtype=dtype, device=device)
        self.compute = compute or _default_compute

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
        return self.gathered.view(self.H, self.B, self.S, self.D).permute(1, 0, 2, 3)

    def _compute_chunk(self, c, q, k, v, causal, scale):
        # this rank's [h, B, S, D] slot seen as [B, h, S, D]
        self.compute(q, k, v, causal=causal, scale=scale,
                     out=self.gathered[c, self.rank].permute(1, 0, 2, 3))

    def compute_local(self, qs: Sequence[torch.Tensor], ks: Sequence[torch.Tensor],
                      vs: Sequence[torch.Tensor], *, causal: bool = True,
                      scale: float | None = None) -> None:
        """This rank's heads only, no collective."""
        for c in range(self.chunks):
            self._compute_chunk(c, qs[c], ks[c], vs[c], causal, scale)

    def __call__(self, qs: Sequence[torch.Tensor], ks: Sequence[torch.Tensor],
                 vs: Sequence[torch.Tensor], *, causal: bool = True,
                 scale: float | None = None) -> torch.Tensor:
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
