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


def _rank_major(buf: torch.Tensor, shape, world: int) -> torch.Tensor:
    """[world * B, Lr, ...] gathered shards as [B, world * Lr, ...] (rank order)."""
    B, Lr = shape[0], shape[1]
    buf = buf.view((world,) + tuple(shape))
    if B == 1:
        return buf.view((1, world * Lr) + tuple(shape[2:]))
    return buf.transpose(0, 1).reshape((B, world * Lr) + tuple(shape[2:]))


def gather_sequence(t: torch.Tensor, group, world: int) -> torch.Tensor:
    """All-gather [B, Lr, ...] shards along dim 1 into [B, world * Lr, ...] (rank order)."""
    t = t.contiguous()
    buf = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), device=t.device, dtype=t.dtype)
    dist.all_gather_into_tensor(buf, t, group=group)
    return _rank_major(buf, t.shape, world)


def allreduce_sum(t: torch.Tensor, group) -> torch.Tensor:
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


class QueryShards:
    """The layer's view of its process group and of its share of the query sequence.

    ``layout="contiguous"``: rank r owns tokens [r*n, (r+1)*n) (n = the local length).
    ``layout="zigzag"``: the sequence is cut into 2·P·folds equal segments, dealt to the ranks in
    sweeps that alternate direction (0..P-1, P-1..0, 0..P-1, ...); rank r owns its 2·folds
    segments in sequence order.  With folds = 1 rank r owns segments r and 2P-1-r: every rank gets
    the same number of causal (query, key) pairs, where contiguous blocks give the last rank
    (2P-1)/P^2 of the indexer work.  More folds also even out costs that grow non-linearly along
    the sequence -- the adaptive k_t, hence the SDPA work, rises with the position (at 128K tokens
    on 8 ranks the busiest rank's SDPA keys are 1.15x the mean with 1 fold, 1.02x with 4).  Zigzag
    takes a single sequence per call (batch 1)."""

    def __init__(self, group, layout: str = "contiguous", folds: int = 1):
        if layout not in ("contiguous", "zigzag"):
            raise ValueError(f"unknown layout {layout!r}")
        if folds < 1:
            raise ValueError("folds must be >= 1")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.layout = layout
        self.folds = folds
        self._side = None   # stream of the asynchronous gathers' reordering
        self._perm = {}     # (device, world, segments per rank) -> segment permutation

    def segments(self, L_local: int):
        """[(local_start, length, absolute_position_of_first_token)] of this rank's tokens."""
        if self.layout == "contiguous":
            return [(0, L_local, self.rank * L_local)]
        nseg = 2 * self.folds
        if L_local % nseg:
            raise ValueError(f"zigzag sharding needs a multiple of {nseg} local tokens")
        S = L_local // nseg
        return [(k * S, S, zigzag_block(k, self.world, self.rank) * S) for k in range(nseg)]

    def positions(self, L_local: int, device) -> torch.Tensor:
        return torch.cat([torch.arange(p0, p0 + n, device=device) for _, n, p0 in self.segments(L_local)])

    def start(self, L_local: int) -> int:
        return self.segments(L_local)[0][2]

    def gather(self, t: torch.Tensor) -> torch.Tensor:
        """All-gather every rank's [B, L_local, ...] tokens into [B, L_total, ...] in sequence order."""
        t = t.contiguous()
        buf = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), device=t.device, dtype=t.dtype)
        dist.all_gather_into_tensor(buf, t, group=self.group)
        return self._sequence_order(buf, t)

    def gather_async(self, t: torch.Tensor):
        """Start the all-gather of :meth:`gather` and return ``finish()``, which makes the current
        stream wait for it and returns the same tensor.  The collective runs on NCCL's stream
        meanwhile, so work queued in between (the indexer, for K and V) overlaps the transfer; on
        CUDA the reordering into sequence order follows the collective on a side stream, so it
        overlaps that work too."""
        t = t.contiguous()
        buf = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), device=t.device, dtype=t.dtype)
        work = dist.all_gather_into_tensor(buf, t, group=self.group, async_op=True)
        if not t.is_cuda or self.layout == "contiguous":
            def finish():
                work.wait()
                return self._sequence_order(buf, t)
            return finish
        main = torch.cuda.current_stream(t.device)
        if self._side is None:
            self._side = torch.cuda.Stream(device=t.device)
        side = self._side
        side.wait_stream(main)  # buf and t were made on the main stream
        with torch.cuda.stream(side):
            work.wait()  # the side stream waits for the collective
            out = self._sequence_order(buf, t)
            done = torch.cuda.Event()
            done.record(side)
        buf.record_stream(side)

        def finish():
            main.wait_event(done)
            out.record_stream(main)
            return out

        return finish

    def _sequence_order(self, g: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        """The gathered shards ([world * B, L_local, ...] in rank order) in sequence order: one
        gather copy of whole segments (zigzag) or a view (contiguous blocks)."""
        if self.layout == "contiguous":
            return g if g.shape[0] == t.shape[0] else _rank_major(g, t.shape, self.world)
        B, Ll = t.shape[0], t.shape[1]
        nseg = 2 * self.folds
        S = Ll // nseg
        rest = tuple(t.shape[2:])
        # rank-major segment r * nseg + k is rank r's k-th segment; sequence segment j = k * P + i
        # belongs to sweep k, owned by rank i (even k) or P-1-i (odd k)
        key = (g.device, self.world, nseg)
        perm = self._perm.get(key)
        if perm is None:
            order = []
            for j in range(self.world * nseg):
                k, i = divmod(j, self.world)
                r = i if k % 2 == 0 else self.world - 1 - i
                order.append(r * nseg + k)
            perm = torch.tensor(order, dtype=torch.long, device=g.device)
            self._perm[key] = perm
        blocks = g.view((self.world * nseg, S) + rest) if B == 1 else \
            _rank_major(g, t.shape, self.world).view((B, self.world * nseg, S) + rest)
        if B == 1:
            return blocks.index_select(0, perm).view((1, self.world * Ll) + rest)
        return blocks.index_select(1, perm).view((B, self.world * Ll) + rest)

    def allreduce(self, t):
        return allreduce_sum(t, self.group)


class SequenceShards:
    """The layer's view of a process group whose ranks each hold different sequences of the
    batch (decode with the KV cache sharded by sequence).  Nothing is exchanged but the
    adaptive k's two fp64 numbers: its variance mean runs over every (batch, query) row of the
    call (adaptive_topk.py:93-96), so over all ranks' sequences."""

    def __init__(self, group):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def allreduce(self, t):
        return allreduce_sum(t, self.group)


def enable_sequence_sharding(layer, group=None):
    """Make ``layer`` run its batch sharded by sequence over ``group``: each rank passes its own
    sequences (and their KV cache); the selections equal those of one call over all sequences."""
    layer.sequence_shards = SequenceShards(group if group is not None else dist.group.WORLD)
    return layer


def zigzag_block(k: int, world: int, rank: int) -> int:
    """Sequence index of rank's k-th zigzag segment (segments of L / (2 * world * folds) tokens)."""
    return k * world + (rank if k % 2 == 0 else world - 1 - rank)


def zigzag_slice(x: torch.Tensor, world: int, rank: int, folds: int = 1) -> torch.Tensor:
    """This rank's tokens of a full [B, L, ...] sequence under the zigzag layout."""
    L = x.shape[1]
    nseg = 2 * folds
    if L % (nseg * world):
        raise ValueError(f"sequence length {L} does not split into {nseg * world} segments")
    S = L // (nseg * world)
    return torch.cat([x[:, zigzag_block(k, world, rank) * S:(zigzag_block(k, world, rank) + 1) * S]
                      for k in range(nseg)], dim=1)


def enable_query_sharding(layer, group=None, layout: str = "contiguous", folds: int = 1):
    """Make ``layer`` (a GatedSparseAttention) run query-sharded over ``group``: its input is
    this rank's tokens (a contiguous block, or for ``layout="zigzag"`` the segments given by
    :func:`zigzag_slice` with the same ``folds``) and its output the same tokens."""
    layer.query_shards = QueryShards(group if group is not None else dist.group.WORLD, layout, folds)
    return layer
