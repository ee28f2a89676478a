"""Query-sequence sharding on CPU ranks (gloo, world size 2): the decomposition the layer uses
across GPUs (gsa_b200.sharded) -- contiguous query blocks, an all-gather of K / V / k^I, an
offset-causal indexer and an all-reduce of the variance sum -- reproduces the unsharded layer,
and so does the batch split by sequence (the decode layout: only the variance sum is shared).
The kernels' roles are played by the CPU oracle; the sharding code is the product's.  Also:
a rank that fails before the exchange makes the other rank's collective end with an error
instead of waiting forever."""

import datetime
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT, golden_inputs, load_golden  # noqa: F401


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _sharded_oracle_layer(W, cfg, x_local, sp):
    """The layer's sharded forward with oracle stand-ins for the kernels."""
    import torch.nn.functional as F
    import gsa_oracle as O

    B, Lr, _ = x_local.shape
    segs = sp.segments(Lr)
    oc = O.OracleConfig.from_config(cfg)
    pos = sp.positions(Lr, "cpu").unsqueeze(0).expand(B, -1)
    cos, sin = O.rope_cache(cfg.d_head, cfg.max_position_embeddings, cfg.rope_base, cfg.rope_scaling)
    q, k, v = O.project(W, oc, x_local, pos, cos, sin)
    q_idx = F.linear(x_local, W["indexer.q_proj.weight"]).view(B, Lr, cfg.n_indexer_heads, cfg.d_indexer)
    k_idx = F.linear(x_local, W["indexer.k_proj.weight"])
    wts = torch.sigmoid(F.linear(x_local, W["indexer.weight_proj.weight"], W["indexer.weight_proj.bias"]))
    # exchange: keys of every rank, in sequence order
    k_all, v_all, kI_all = sp.gather(k), sp.gather(v), sp.gather(k_idx)
    L = kI_all.shape[1]
    scores = torch.cat([O.indexer_scores_from_proj(q_idx[:, l0:l0 + n], kI_all, wts[:, l0:l0 + n],
                                                   W["indexer.bias"], "sigmoid", q_offset=p0)
                        for l0, n, p0 in segs], dim=1)
    var, valid = O.row_variance(scores)
    total = sp.allreduce(torch.tensor([float(var.double().sum()), float(var.numel())], dtype=torch.float64))
    mean = torch.tensor(float(total[0]) / float(total[1]), dtype=var.dtype)
    kv = O.adaptive_k(var, valid, mean, cfg.k_base, cfg.k_min, cfg.k_max, cfg.adaptive_k_temperature)
    idx, msk = O.topk_select(scores, min(cfg.k_max, L), kv)
    attn, _ = O.sparse_attention(q, k_all, v_all, idx, msk, cfg.n_heads // cfg.n_kv_heads,
                                 1.0 / math.sqrt(cfg.d_head))
    g = F.linear(x_local, W["output_gate.gate_proj.weight"], W["output_gate.gate_proj.bias"])
    gated = attn * torch.sigmoid(g.view(B, Lr, cfg.n_heads, cfg.d_head))
    return F.linear(gated.reshape(B, Lr, -1), W["o_proj.weight"]), kv


def _worker_equivalence(rank, world, port, layout, folds, q):
    import sys
    for p in (ROOT / "gated-sparse-attention_b200", ROOT / "oracle", ROOT / "tests"):
        sys.path.insert(0, str(p))
    torch.set_num_threads(1)
    from gsa_b200.sharded import QueryShards, shard_bounds, zigzag_slice
    import gsa_oracle as O

    try:
        _init(rank, world, port)
        _, meta = load_golden("tiny_fp32_b2_l192")
        cfg, m, x = golden_inputs(meta)
        x = x[:1]  # one sequence (the zigzag layout takes one per call)
        W = dict(m.state_dict())
        L = x.shape[1]
        sp = QueryShards(dist.group.WORLD, layout, folds)
        if layout == "zigzag":
            x_local = zigzag_slice(x, world, rank, folds)
        else:
            s0, s1 = shard_bounds(L, world, rank)
            x_local = x[:, s0:s1]
        out_local, kv_local = _sharded_oracle_layer(W, cfg, x_local.contiguous(), sp)
        out_full = sp.gather(out_local)
        kv_full = sp.gather(kv_local.contiguous())
        if rank == 0:
            ref = O.gsa_forward(W, O.OracleConfig.from_config(cfg), x, chunk=64, keep=("k_values",))
            err = float((out_full - ref["out"]).norm() / ref["out"].norm())
            kdiff = int((kv_full != ref["k_values"]).sum())
            q.put(("ok", err, kdiff))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put(("error", repr(e), -1))


@pytest.mark.parametrize("layout,folds", [("contiguous", 1), ("zigzag", 1), ("zigzag", 3)])
def test_query_sharded_layer_matches_unsharded(layout, folds):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_equivalence, args=(r, 2, port, layout, folds, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    status, err, kdiff = q.get(timeout=10)
    assert status == "ok", err
    assert err < 1e-5, err
    assert kdiff == 0


def _worker_sequence_shards(rank, world, port, q):
    """Each rank runs the oracle layer on its own sequences of the batch; only the variance sum
    is all-reduced (SequenceShards, the decode layout across GPUs)."""
    import sys
    for p in (ROOT / "gated-sparse-attention_b200", ROOT / "oracle", ROOT / "tests"):
        sys.path.insert(0, str(p))
    torch.set_num_threads(1)
    import torch.nn.functional as F
    import gsa_oracle as O
    from gsa_b200.sharded import SequenceShards

    try:
        _init(rank, world, port)
        _, meta = load_golden("tiny_fp32_b2_l192")
        cfg, m, x = golden_inputs(meta)
        W = dict(m.state_dict())
        B, L = x.shape[0], x.shape[1]
        per = B // world
        x_local = x[rank * per:(rank + 1) * per]
        shards = SequenceShards(dist.group.WORLD)
        oc = O.OracleConfig.from_config(cfg)
        pos = torch.arange(L).unsqueeze(0).expand(per, -1)
        cos, sin = O.rope_cache(cfg.d_head, cfg.max_position_embeddings, cfg.rope_base, cfg.rope_scaling)
        qh, k, v = O.project(W, oc, x_local, pos, cos, sin)
        q_idx = F.linear(x_local, W["indexer.q_proj.weight"]).view(per, L, cfg.n_indexer_heads, cfg.d_indexer)
        k_idx = F.linear(x_local, W["indexer.k_proj.weight"])
        wts = torch.sigmoid(F.linear(x_local, W["indexer.weight_proj.weight"], W["indexer.weight_proj.bias"]))
        scores = O.indexer_scores_from_proj(q_idx, k_idx, wts, W["indexer.bias"], "sigmoid", q_offset=0)
        var, valid = O.row_variance(scores)
        total = shards.allreduce(torch.tensor([float(var.double().sum()), float(var.numel())], dtype=torch.float64))
        mean = torch.tensor(float(total[0]) / float(total[1]), dtype=var.dtype)
        kv = O.adaptive_k(var, valid, mean, cfg.k_base, cfg.k_min, cfg.k_max, cfg.adaptive_k_temperature)
        idx, msk = O.topk_select(scores, min(cfg.k_max, L), kv)
        attn, _ = O.sparse_attention(qh, k, v, idx, msk, cfg.n_heads // cfg.n_kv_heads, 1.0 / math.sqrt(cfg.d_head))
        g = F.linear(x_local, W["output_gate.gate_proj.weight"], W["output_gate.gate_proj.bias"])
        out = F.linear((attn * torch.sigmoid(g.view(per, L, cfg.n_heads, cfg.d_head))).reshape(per, L, -1),
                       W["o_proj.weight"])
        outs = [torch.empty_like(out) for _ in range(world)]
        ks = [torch.empty_like(kv) for _ in range(world)]
        dist.all_gather(outs, out)
        dist.all_gather(ks, kv)
        if rank == 0:
            ref = O.gsa_forward(W, oc, x, chunk=64, keep=("k_values",))
            full = torch.cat(outs)
            err = float((full - ref["out"]).norm() / ref["out"].norm())
            q.put(("ok", err, int((torch.cat(ks) != ref["k_values"]).sum())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put(("error", repr(e), -1))


def test_sequence_sharded_batch_matches_unsharded():
    """The batch's sequences split over two ranks (SequenceShards): with the variance sum
    all-reduced, every k_t and output equals the one-process layer over the whole batch."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_sequence_shards, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    status, err, kdiff = q.get(timeout=10)
    assert status == "ok", err
    assert err < 1e-5, err
    assert kdiff == 0


def _worker_async_gather(rank, world, port, q):
    import sys
    for p in (ROOT / "gated-sparse-attention_b200",):
        sys.path.insert(0, str(p))
    from gsa_b200.sharded import QueryShards

    try:
        _init(rank, world, port)
        ok = True
        for layout, folds in (("contiguous", 1), ("zigzag", 1), ("zigzag", 2)):
            sp = QueryShards(dist.group.WORLD, layout, folds)
            t = torch.arange(2 * 8 * 3, dtype=torch.float32).view(2, 8, 3) + 1000 * rank
            t = t[:1] if layout == "zigzag" else t
            finish = sp.gather_async(t)
            ok = ok and torch.equal(finish(), sp.gather(t))
        q.put(("ok", ok) if rank == 0 else ("rank", ok))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put(("error", repr(e)))


def test_async_gather_equals_gather():
    """The asynchronous all-gather the layer uses for K/V returns what the blocking one returns."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_async_gather, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = [q.get(timeout=10) for _ in range(2)]
    assert all(r[0] in ("ok", "rank") and r[1] is True for r in results), results


def _worker_failure(rank, world, port, q):
    import sys
    for p in (ROOT / "gated-sparse-attention_b200",):
        sys.path.insert(0, str(p))
    from gsa_b200.sharded import QueryShards

    _init(rank, world, port, timeout_s=5)
    sp = QueryShards(dist.group.WORLD)
    if rank == 1:
        # this rank fails before the key exchange and never joins it
        os._exit(0)
    try:
        sp.gather(torch.zeros(1, 4, 2))
        q.put("no error")
    except Exception as e:
        q.put("error: " + type(e).__name__)


def test_failed_rank_surfaces_as_collective_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_failure, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    msg = q.get(timeout=10)
    assert msg.startswith("error"), msg


def test_shard_bounds():
    from gsa_b200.sharded import shard_bounds, zigzag_slice

    x = torch.arange(16).view(1, 16)
    assert zigzag_slice(x, 2, 0).tolist() == [[0, 1, 2, 3, 12, 13, 14, 15]]
    assert zigzag_slice(x, 2, 1).tolist() == [[4, 5, 6, 7, 8, 9, 10, 11]]
    # two folds: 8 segments of 2 dealt 0 1 | 1 0 | 0 1 | 1 0
    assert zigzag_slice(x, 2, 0, folds=2).tolist() == [[0, 1, 6, 7, 8, 9, 14, 15]]
    assert zigzag_slice(x, 2, 1, folds=2).tolist() == [[2, 3, 4, 5, 10, 11, 12, 13]]

    assert shard_bounds(131072, 8, 7) == (114688, 131072)
    assert shard_bounds(10, 2, 0) == (0, 5)
    with pytest.raises(ValueError):
        shard_bounds(10, 3, 0)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("folds", [1, 3, 4])
@pytest.mark.parametrize("B", [1, 2])
def test_sequence_order_of_gathered_zigzag_shards(world, folds, B):
    """The gathered shards of every rank (rank order, as all_gather_into_tensor lays them out) put
    back into sequence order equal the full sequence, for the zigzag layout at 2-8 ranks (the
    permutation the 8-GPU runs use) and for contiguous blocks."""
    from gsa_b200.sharded import QueryShards, zigzag_slice

    L = 2 * folds * world * 3
    full = torch.arange(B * L * 2, dtype=torch.float32).view(B, L, 2)
    for layout in ("zigzag", "contiguous"):
        if layout == "zigzag" and B != 1:
            continue
        qs = object.__new__(QueryShards)
        qs.world, qs.layout, qs.folds, qs._perm, qs._side = world, layout, folds, {}, None
        if layout == "zigzag":
            shards = [zigzag_slice(full, world, r, folds) for r in range(world)]
        else:
            shards = [full[:, r * (L // world):(r + 1) * (L // world)] for r in range(world)]
        buf = torch.cat(shards, dim=0)  # [world * B, L_local, 2]
        out = qs._sequence_order(buf, shards[0])
        assert torch.equal(out, full), (layout, world, folds, B)
