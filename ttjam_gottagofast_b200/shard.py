"""Batch sharding of the forward pass over ranks (one process per GPU).

Sequences are independent in the reference forward (attention never crosses
the batch dimension, torch_transformer_benchmark.py:97-117), so a batch splits
into whole sequences with replicated weights and no exchange inside the step.
Two assignments:

* `shard_range`: contiguous slices, sizes differing by at most one;
* `balanced_assignment`: the same number of sequences per rank, chosen so
  that the estimated work -- the projections over each sequence's rows plus
  the attention, which grows with the square of its valid length under the
  causal and key-padding masks -- is as even as a greedy largest-first
  placement makes it. The projections run over all rows, or (with
  `row_tile`, the tensor-core schedule's dead-row tiling) over the row tiles
  up to the last valid key rounded up to 64. The slowest rank sets the step
  time, so this is what evens the ranks out for random lengths.

The only collective is the optional gather of the outputs afterwards
(`all_gather_into_tensor` over NCCL / NVLink on GPUs, gloo on CPU), which pads
uneven slices to a common size, trims after, and undoes the assignment's
order through its index map.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

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


def sequence_cost(length: int, seq_len: int, attn_weight: float = 1.0,
                  row_tile: int = 0) -> float:
    """Relative cost of one sequence, in units of one row's projection work:
    the projections over its rows -- all seq_len of them, or with row_tile > 0
    the tiles of row_tile rows up to its last valid key rounded up to 64 (when
    row_tile divides seq_len, the tiles of one sequence are its own) -- plus
    the causal attention over its valid length (length^2 / 2 query-key pairs),
    each pair weighing attn_weight / seq_len."""
    rows = seq_len
    if row_tile > 0 and seq_len % row_tile == 0:
        live = -(-length // 64) * 64
        rows = min(seq_len, -(-live // row_tile) * row_tile)
    return rows + attn_weight * length * (length + 1) / (2.0 * max(seq_len, 1))


def balanced_assignment(lengths: Sequence[int], world: int, seq_len: Optional[int] = None,
                        attn_weight: float = 1.0, row_tile: int = 0) -> List[List[int]]:
    """Sequence indices per rank: as many per rank as `shard_range` gives
    (sizes differ by at most one), placed largest `sequence_cost` first onto
    the rank with the least cost so far among those with room; each rank's
    indices in ascending order. Deterministic: ties go to the lower rank, then
    the lower index."""
    if world <= 0:
        raise ValueError("world must be positive")
    n = len(lengths)
    s = int(seq_len if seq_len is not None else (max(lengths) if n else 0))
    caps = [shard_range(n, world, r)[1] for r in range(world)]
    cost = [sequence_cost(int(l), s, attn_weight, row_tile) for l in lengths]
    order = sorted(range(n), key=lambda i: (-cost[i], i))
    load = [0.0] * world
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min((r for r in range(world) if len(out[r]) < caps[r]), key=lambda r: (load[r], r))
        out[r].append(i)
        load[r] += cost[i]
    return [sorted(ix) for ix in out]


def sharded_forward(forward: Callable[[torch.Tensor, Optional[torch.Tensor]], torch.Tensor],
                    x: torch.Tensor, mask: Optional[torch.Tensor] = None,
                    group=None, gather: bool = True,
                    assignment: Optional[List[List[int]]] = None) -> torch.Tensor:
    """Run `forward` on this rank's sequences of the batch; with `gather`,
    return the full [B, S, D] output on every rank in the original sequence
    order, else this rank's part.

    `x` and `mask` are the full batch (every rank holds the same inputs, as in
    the reference's seeded generation); `forward` is typically a
    `UserOptimizedTransformer` on this rank's GPU. `assignment` (one index
    list per rank, e.g. from `balanced_assignment`) replaces the contiguous
    `shard_range` slices; every rank must pass the same one.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    b = x.shape[0]
    if assignment is None:
        assignment = [list(range(*_as_range(shard_range(b, world, r)))) for r in range(world)]
    if len(assignment) != world or sorted(i for ix in assignment for i in ix) != list(range(b)):
        raise ValueError("assignment must give every sequence to exactly one of the ranks")
    mine = assignment[rank]
    contiguous = not mine or mine == list(range(mine[0], mine[0] + len(mine)))
    if contiguous:
        start = mine[0] if mine else 0
        xs = x[start:start + len(mine)]
        ms = None if mask is None else mask[start:start + len(mine)]
    else:
        idx = torch.tensor(mine, device=x.device)
        xs = x.index_select(0, idx)
        ms = None if mask is None else mask.index_select(0, idx)
    y_local = forward(xs, ms) if mine else x[:0].clone()
    if not gather or world == 1:
        return y_local
    per = max(len(ix) for ix in assignment)  # every rank sends a slice of this size
    send = y_local.new_zeros((per,) + tuple(x.shape[1:]))
    send[:len(mine)] = y_local
    recv = y_local.new_empty((per * world,) + tuple(x.shape[1:]))
    dist.all_gather_into_tensor(recv, send, group=group)
    # row r*per + k of recv is sequence assignment[r][k]
    src = torch.empty(b, dtype=torch.long)
    for r, ix in enumerate(assignment):
        for k, i in enumerate(ix):
            src[i] = r * per + k
    return recv.index_select(0, src.to(recv.device))


def _as_range(start_count: Tuple[int, int]) -> Tuple[int, int]:
    start, count = start_count
    return start, start + count
