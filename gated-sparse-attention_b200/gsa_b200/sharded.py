"""Query-sequence sharding of one GSA layer over several GPUs (one process per GPU).

Rank r of P owns the contiguous query block [r * L/P, (r+1) * L/P) of every sequence and
projects only its own tokens.  The layer then needs two exchanges:

  * an all-gather of the post-RoPE K, the post-G2 V and the indexer keys k^I, so that every
    rank can score and attend to all earlier keys (its queries are masked offset-causally);
  * an all-reduce of (sum of per-row variances, row count): the adaptive k divides each row's
    variance by the mean over every (batch, query) row of the layer call
    (adaptive_topk.py:93-96), so the mean spans all ranks.

The candidate selection (the k_max best keys per row) does not depend on that mean, so each rank
selects locally and only the final truncation to k_t waits for the all-reduce.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(L_total: int, world: int, rank: int):
    """[start, end) of rank's contiguous query block; L_total must divide evenly."""
    if L_total % world:
        raise ValueError(f"sequence length {L_total} does not divide over {world} ranks")
    n = L_total // world
    return rank * n, (rank + 1) * n


def gather_sequence(t: torch.Tensor, group, world: int) -> torch.Tensor:
    """All-gather [B, Lr, ...] shards along dim 1 into [B, world * Lr, ...] (rank order)."""
    t = t.contiguous()
    B, Lr = t.shape[0], t.shape[1]
    buf = torch.empty((world * B,) + tuple(t.shape[1:]), device=t.device, dtype=t.dtype)
    dist.all_gather_into_tensor(buf, t, group=group)
    buf = buf.view((world,) + tuple(t.shape))
    if B == 1:
        return buf.view((1, world * Lr) + tuple(t.shape[2:]))
    return buf.transpose(0, 1).reshape((B, world * Lr) + tuple(t.shape[2:]))


def allreduce_sum(t: torch.Tensor, group) -> torch.Tensor:
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


class QueryShards:
    """The layer's view of its process group."""

    def __init__(self, group):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def start(self, L_local: int) -> int:
        return self.rank * L_local

    def gather(self, t):
        return gather_sequence(t, self.group, self.world)

    def allreduce(self, t):
        return allreduce_sum(t, self.group)


def enable_query_sharding(layer, group=None):
    """Make ``layer`` (a GatedSparseAttention) run query-sharded over ``group``: its input is
    this rank's block of tokens and its output the same block."""
    layer.query_shards = QueryShards(group if group is not None else dist.group.WORLD)
    return layer
