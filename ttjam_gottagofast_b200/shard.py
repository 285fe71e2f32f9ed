"""Batch sharding of the forward pass over ranks (one process per GPU).

Sequences are independent in the reference forward (attention never crosses
the batch dimension, torch_transformer_benchmark.py:97-117), so a batch splits
into contiguous slices of whole sequences with replicated weights and no
exchange inside the step. The only collective is the optional gather of the
outputs afterwards (`all_gather_into_tensor` over NCCL / NVLink on GPUs, gloo
on CPU), which pads uneven slices to a common size and trims after.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist


def shard_range(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous slice [start, start+count) of `batch` sequences owned by
    `rank`; slice sizes differ by at most one, earlier ranks take the extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if batch < 0:
        raise ValueError("batch must be >= 0")
    base, extra = divmod(batch, world)
    count = base + (1 if rank < extra else 0)
    start = rank * base + min(rank, extra)
    return start, count


def sharded_forward(forward: Callable[[torch.Tensor, Optional[torch.Tensor]], torch.Tensor],
                    x: torch.Tensor, mask: Optional[torch.Tensor] = None,
                    group=None, gather: bool = True) -> torch.Tensor:
    """Run `forward` on this rank's slice of the batch; with `gather`, return the
    full [B, S, D] output on every rank in the original sequence order, else
    this rank's slice.

    `x` and `mask` are the full batch (every rank holds the same inputs, as in
    the reference's seeded generation); `forward` is typically a
    `UserOptimizedTransformer` on this rank's GPU.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    b = x.shape[0]
    start, count = shard_range(b, world, rank)
    xs = x[start:start + count]
    ms = None if mask is None else mask[start:start + count]
    y_local = forward(xs, ms) if count > 0 else x[:0].clone()
    if not gather or world == 1:
        return y_local
    per = -(-b // world)  # ceil: every rank contributes a slice of this size
    send = y_local.new_zeros((per,) + tuple(x.shape[1:]))
    send[:count] = y_local
    recv = y_local.new_empty((per * world,) + tuple(x.shape[1:]))
    dist.all_gather_into_tensor(recv, send, group=group)
    parts = []
    for r in range(world):
        s_r, c_r = shard_range(b, world, r)
        parts.append(recv[r * per:r * per + c_r])
    return torch.cat(parts, 0)
