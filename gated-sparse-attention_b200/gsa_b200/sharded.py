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
    """The layer's view of its process group and of its share of the query sequence.

    ``layout="contiguous"``: rank r owns tokens [r*n, (r+1)*n) (n = the local length).
    ``layout="zigzag"``: the sequence is cut into 2P equal segments and rank r owns segments r and
    2P-1-r, in that order, so every rank gets the same number of causal (query, key) pairs --
    with contiguous blocks the last rank does (2P-1)/P^2 of the indexer work.  Zigzag takes a
    single sequence per call (batch 1)."""

    def __init__(self, group, layout: str = "contiguous"):
        if layout not in ("contiguous", "zigzag"):
            raise ValueError(f"unknown layout {layout!r}")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.layout = layout

    def segments(self, L_local: int):
        """[(local_start, length, absolute_position_of_first_token)] of this rank's tokens."""
        if self.layout == "contiguous":
            return [(0, L_local, self.rank * L_local)]
        if L_local % 2:
            raise ValueError("zigzag sharding needs an even number of local tokens")
        S = L_local // 2
        return [(0, S, self.rank * S), (S, S, (2 * self.world - 1 - self.rank) * S)]

    def positions(self, L_local: int, device) -> torch.Tensor:
        return torch.cat([torch.arange(p0, p0 + n, device=device) for _, n, p0 in self.segments(L_local)])

    def start(self, L_local: int) -> int:
        return self.segments(L_local)[0][2]

    def gather(self, t: torch.Tensor) -> torch.Tensor:
        """All-gather every rank's [B, L_local, ...] tokens into [B, L_total, ...] in sequence order."""
        g = gather_sequence(t, self.group, self.world)
        if self.layout == "contiguous":
            return g
        B, Ll = t.shape[0], t.shape[1]
        S = Ll // 2
        rest = tuple(t.shape[2:])
        blocks = g.view((B, self.world, 2, S) + rest)
        first = blocks[:, :, 0].reshape((B, self.world * S) + rest)            # segments 0..P-1
        second = blocks[:, :, 1].flip(1).reshape((B, self.world * S) + rest)   # segments P..2P-1
        return torch.cat([first, second], dim=1)

    def allreduce(self, t):
        return allreduce_sum(t, self.group)


def zigzag_slice(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's tokens of a full [B, L, ...] sequence under the zigzag layout."""
    L = x.shape[1]
    if L % (2 * world):
        raise ValueError(f"sequence length {L} does not split into {2 * world} segments")
    S = L // (2 * world)
    a, b = rank, 2 * world - 1 - rank
    return torch.cat([x[:, a * S:(a + 1) * S], x[:, b * S:(b + 1) * S]], dim=1)


def enable_query_sharding(layer, group=None, layout: str = "contiguous"):
    """Make ``layer`` (a GatedSparseAttention) run query-sharded over ``group``: its input is
    this rank's tokens (a contiguous block, or for ``layout="zigzag"`` the two segments given by
    :func:`zigzag_slice`) and its output the same tokens."""
    layer.query_shards = QueryShards(group if group is not None else dist.group.WORLD, layout)
    return layer
