"""Query-sequence sharding on 2 GPUs (NCCL): the sharded layer's output, gathered, equals the
1-GPU layer's output on the same input; a batch split by sequence (prefill into the cache, then
decode steps) equals the 1-GPU batch.  Skipped unless two CUDA devices are visible."""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT

pytestmark = pytest.mark.gpu

CFG = dict(d_model=1024, n_heads=8, n_kv_heads=2, d_indexer=64, n_indexer_heads=8, k_base=128,
           k_min=64, k_max=256, max_position_embeddings=8192)
L = 4096


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, layout, folds, q):
    import sys
    sys.path.insert(0, str(ROOT / "gated-sparse-attention_b200"))
    import torch.distributed as dist
    from gsa_b200 import GSAConfig, GatedSparseAttention
    from gsa_b200.sharded import enable_query_sharding, zigzag_slice

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        cfg = GSAConfig(**CFG)
        torch.manual_seed(0)
        m = GatedSparseAttention(cfg).eval().to(torch.bfloat16).cuda()
        gen = torch.Generator().manual_seed(1)
        x = torch.randn(1, L, cfg.d_model, generator=gen).to(torch.bfloat16).cuda()
        with torch.no_grad():
            ref = m(x)[0] if rank == 0 else None
            enable_query_sharding(m, dist.group.WORLD, layout, folds)
            Lr = L // world
            x_local = zigzag_slice(x, world, rank, folds) if layout == "zigzag" else x[:, rank * Lr:(rank + 1) * Lr]
            out = m(x_local.contiguous())[0]
            full = m.query_shards.gather(out)
        torch.cuda.synchronize()
        if rank == 0:
            err = float((full.double() - ref.double()).norm() / ref.double().norm())
            q.put(("ok", err))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put(("error", repr(e)))


@pytest.mark.parametrize("layout,folds", [("contiguous", 1), ("zigzag", 1), ("zigzag", 4)])
def test_two_gpu_query_sharding_matches_single_gpu(layout, folds):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, layout, folds, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    status, val = q.get(timeout=30)
    assert status == "ok", val
    # same kernels on the same rows: only the fp64 atomic order of the row statistics and the
    # all-reduced variance sum can differ, which can move a k_t boundary
    assert val < 1e-2, val


def _worker_decode(rank, world, port, q):
    """Sequence-sharded prefill + decode (the native step in two phases around the variance
    all-reduce) against one process holding every sequence."""
    import sys
    sys.path.insert(0, str(ROOT / "gated-sparse-attention_b200"))
    import torch.distributed as dist
    from gsa_b200 import GSAConfig, GatedSparseAttention
    from gsa_b200.sharded import enable_sequence_sharding

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        cfg = GSAConfig(**CFG)
        torch.manual_seed(0)
        m = GatedSparseAttention(cfg).eval().to(torch.bfloat16).cuda()
        B, Lp, steps = 4, 1500, 3
        gen = torch.Generator().manual_seed(3)
        x = torch.randn(B, Lp + steps, cfg.d_model, generator=gen).to(torch.bfloat16).cuda()

        def run(xs):
            n = xs.shape[0]
            outs = []
            with torch.no_grad():
                out, c, _ = m(xs[:, :Lp], past_key_value=m.allocate_cache(n, Lp + steps), use_cache=True)
                outs.append(out)
                for s in range(steps):
                    out, c, _ = m(xs[:, Lp + s:Lp + s + 1], past_key_value=c, use_cache=True)
                    outs.append(out)
            return torch.cat(outs, 1)

        ref = run(x) if rank == 0 else None
        enable_sequence_sharding(m, dist.group.WORLD)
        per = B // world
        mine = run(x[rank * per:(rank + 1) * per].contiguous())
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        torch.cuda.synchronize()
        if rank == 0:
            full = torch.cat(parts)
            q.put(("ok", float((full.double() - ref.double()).norm() / ref.double().norm())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put(("error", repr(e)))


def test_two_gpu_sequence_sharded_decode_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker_decode, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    status, val = q.get(timeout=30)
    assert status == "ok", val
    # the GEMMs run on half the rows and the variance sum is all-reduced in another order
    assert val < 1e-2, val
