"""Head-sharded multi-GPU causal prefill with an all-gather of the output.

Every (batch, head) pair of attention is independent, so G ranks (one process
per GPU) split the heads evenly -- rank r owns heads [r*H/G, (r+1)*H/G) for
every batch entry -- and compute them with no exchange.  The only collective
is one all-gather of O.  Each rank writes its heads into a head-major local
buffer [H/G, B, S, D]; the gather lands in [G, H/G, B, S, D], which is exactly
a strided [B, H, S, D] view (no copy):

    gathered.view(G*H/G, B, S, D).permute(1, 0, 2, 3)  ->  [B, H, S, D]

The collective goes through ``torch.distributed`` (NCCL over NVLink on GPUs,
gloo on CPU for the tests).  The per-rank compute is injectable so that the
shard/gather logic can be tested on CPU ranks against the oracle.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist


def head_range(heads: int, world: int, rank: int) -> tuple[int, int]:
    """Heads owned by `rank` of `world` (an even split; heads % world must be 0)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if heads % world:
        raise ValueError(f"{heads} heads cannot be split evenly over {world} ranks")
    per = heads // world
    return rank * per, (rank + 1) * per


ComputeFn = Callable[..., torch.Tensor]


def _default_compute(q, k, v, *, causal, scale, out):
    from .warpforth import attention

    return attention(q, k, v, causal=causal, scale=scale, out=out)


class ShardedPrefill:
    """Runs this rank's share of a [B, H, S, D] attention and all-gathers O.

    ``local_out`` ([H/G, B, S, D]) and ``gathered`` ([G, H/G, B, S, D]) are
    allocated once and reused.  ``__call__`` takes this rank's q/k/v head
    slices as [B, H/G, S, D] views (any strides) and returns the full output
    as a [B, H, S, D] view of ``gathered``.
    """

    def __init__(self, batch: int, heads: int, seq: int, head_dim: int, *,
                 dtype: torch.dtype, device: torch.device, group=None,
                 compute: ComputeFn | None = None) -> None:
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.h0, self.h1 = head_range(heads, self.world, self.rank)
        self.B, self.H, self.S, self.D = batch, heads, seq, head_dim
        hs = self.h1 - self.h0
        self.gathered = torch.empty((self.world, hs, batch, seq, head_dim), dtype=dtype,
                                    device=device)
        # This rank's slot of the gather buffer: the all-gather runs in place.
        self.local_out = self.gathered[self.rank]
        self.compute = compute or _default_compute

    def shard(self, t: torch.Tensor) -> torch.Tensor:
        """This rank's head slice of a full [B, H, S, D] tensor (a view)."""
        return t[:, self.h0:self.h1]

    def output_view(self) -> torch.Tensor:
        return self.gathered.view(self.H, self.B, self.S, self.D).permute(1, 0, 2, 3)

    def compute_local(self, q, k, v, *, causal: bool = True, scale: float | None = None):
        # [H/G, B, S, D] buffer seen as [B, H/G, S, D]
        return self.compute(q, k, v, causal=causal, scale=scale,
                            out=self.local_out.permute(1, 0, 2, 3))

    def gather(self) -> torch.Tensor:
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered.view(-1), self.local_out.reshape(-1),
                                        group=self.group)
        return self.output_view()

    def __call__(self, q, k, v, *, causal: bool = True, scale: float | None = None):
        self.compute_local(q, k, v, causal=causal, scale=scale)
        return self.gather()
