"""Batch sharding across GPUs (one process per GPU).

ALPHABET rows are independent — every reduction of the forward pass is per
row — so a batch splits across ranks with no collective on the data path:
each rank runs its contiguous slice of rows, and only the final logits are
gathered (when the caller wants them on every rank).  With NCCL over
NVLink/NVSwitch the gather is the only communication; with ``gloo`` the same
code runs on CPU ranks (tests).
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist


def shard_bounds(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced row range [start, stop) of `rank` (first ranks get one extra row)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of world {world}")
    if batch < 0:
        raise ValueError("batch must be non-negative")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(t: torch.Tensor | None, world: int, rank: int) -> torch.Tensor | None:
    if t is None:
        return None
    start, stop = shard_bounds(t.shape[0], world, rank)
    return t[start:stop]


def sharded_forward(forward: Callable[..., torch.Tensor], inputs: torch.Tensor, *,
                    time_delta: torch.Tensor | None = None,
                    observation_mask: torch.Tensor | None = None,
                    valid_mask: torch.Tensor | None = None, group=None,
                    gather: bool = True) -> torch.Tensor:
    """Run `forward` on this rank's rows of the full request and, if `gather`,
    return the outputs of the whole batch on every rank (row order preserved):
    logits [B, K] of a B200Alphabet, or the [B, T, D] output of a
    B200PoleResidueTemporalMixing, whose rows are independent as well."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    meta = {name: shard_rows(t, world, rank) for name, t in
            (("time_delta", time_delta), ("observation_mask", observation_mask),
             ("valid_mask", valid_mask)) if t is not None}
    # metadata keywords only when given, so modules without them (the Laplace
    # layer's forward(inputs)) shard the same way
    local = forward(shard_rows(inputs, world, rank).contiguous(), **meta)
    if not gather or world == 1:
        return local
    batch = inputs.shape[0]
    most = shard_bounds(batch, world, 0)[1]  # the largest shard
    padded = local.new_zeros((most, *local.shape[1:]))
    padded[: local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    out = []
    for r in range(world):
        start, stop = shard_bounds(batch, world, r)
        out.append(parts[r][: stop - start])
    return torch.cat(out, dim=0)


__all__ = ["shard_bounds", "shard_rows", "sharded_forward"]
