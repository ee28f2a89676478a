"""Decode against the append-in-place KV cache.

Indexer: the decode kernel (a few tokens of each of B sequences against their cached keys, one
launch) against the indexer formula (gated_indexer.py:126-153) in fp32, with k^I read through a
cache view (batch stride larger than the key count) and q^I through a row-strided projection
view; against the tensor-core prefill kernel on the same query rows (the same epilogue
arithmetic, with the heads summed in another order).

SDPA: few rows split each row's keys over several CTAs; the merged result against the unsplit
kernel and fp32 attention.

Cache: a prefill into a preallocated cache equals the prefill without one bit for bit; decode
steps append in place (same storage), a second continuation of one cache moves to a new store
and leaves the first continuation intact, a full store grows, and every variant gives the same
outputs as the others bit for bit."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _oracle_scores(qI, kI, w, bias, HI, dI, q_pos0, causal):
    """The indexer formula (gated_indexer.py:126-153) in fp32 on the same (bf16-valued) inputs."""
    B, Lq, _ = qI.shape
    Lkv = kI.shape[1]
    q = qI.float().view(B, Lq, HI, dI)
    raw = torch.einsum("bqhd,bkd->bhqk", q, kI.float()) / math.sqrt(dI)
    s = (torch.sigmoid(raw + bias.view(1, -1, 1, 1)) * w.permute(0, 2, 1).unsqueeze(-1)).sum(1)
    if causal:
        t = torch.arange(Lq).view(-1, 1) + q_pos0
        s = s.masked_fill((torch.arange(Lkv).view(1, -1) > t).unsqueeze(0), float("-inf"))
    return s


def _strided_inputs(B, Lq, Lkv, HI, seed, cap_extra=200, qi_pad=72):
    """qI as a column slice of a wider projection row; kI as the first Lkv slots of a cache
    buffer with room for cap_extra more keys."""
    dI = 64
    g = torch.Generator().manual_seed(seed)
    proj = (torch.randn(B, Lq, HI * dI + qi_pad, generator=g) * 1.3).to(torch.bfloat16)
    store = (torch.randn(B, Lkv + cap_extra, dI, generator=g) * 1.4).to(torch.bfloat16)
    w = torch.sigmoid(torch.randn(B, Lq, HI, generator=g) * 0.3)
    bias = torch.randn(HI, generator=g) * 0.1
    proj, store = proj.to(DEV), store.to(DEV)
    qI = proj[..., 8:8 + HI * dI]
    kI = store[:, :Lkv]
    return qI, kI, w.to(DEV), bias.to(DEV)


@pytest.mark.parametrize("B,Lq,Lkv,HI,causal", [
    (5, 1, 4097, 8, True),
    (3, 3, 2500, 8, True),     # a few tokens per sequence (four column blocks)
    (4, 2, 777, 4, False),     # H_I = 4: two tokens share one column block
    (2, 7, 300, 4, True),
    (64, 1, 20000, 8, True),   # many sequences in one launch
    (2, 1, 1, 8, True),        # a single cached key
])
def test_decode_indexer_matches_oracle(cuda_ok, B, Lq, Lkv, HI, causal):
    from gsa_b200 import ops

    dI = 64
    qI, kI, w, bias = _strided_inputs(B, Lq, Lkv, HI, seed=Lkv + Lq)
    assert kI.stride(0) > Lkv * dI and qI.stride(1) > HI * dI
    dims = ops.make_dims(4096, 32, 8, 128, HI, dI)
    q_pos0 = Lkv - Lq if causal else 0
    stats = torch.zeros(B * Lq, 3, device=DEV, dtype=torch.float64)
    ours = ops.indexer_scores(dims, qI, kI, w, bias, 1 / math.sqrt(dI), q_pos0=q_pos0, causal=causal,
                              row_stats=stats)
    torch.cuda.synchronize()
    ops.check_device_error()
    ref = _oracle_scores(qI.cpu(), kI.cpu(), w.cpu(), bias.cpu(), HI, dI, q_pos0, causal)
    ours = ours.cpu()
    inf = torch.isinf(ref)
    assert torch.equal(torch.isinf(ours), inf)
    err = (ours[~inf] - ref[~inf]).abs() / ref[~inf].abs()
    assert float(err.max()) < 2e-2, float(err.max())
    assert float(err.mean()) < 2e-3
    valid = ~inf.view(B * Lq, Lkv)
    r = ref.view(B * Lq, Lkv).double()
    st = stats.cpu()
    assert torch.equal(st[:, 2], valid.sum(-1).double())
    assert torch.allclose(st[:, 0], torch.where(valid, r, torch.zeros_like(r)).sum(-1), rtol=2e-3, atol=1e-3)


@pytest.mark.parametrize("HI", [8, 4])
def test_decode_indexer_agrees_with_tensor_core_indexer(cuda_ok, HI):
    """The last query row scored by the decode kernel (Lq = 1) and by the tensor-core kernel
    (as the end of a 64-row block): the same epilogue arithmetic on fp32 accumulators of the
    same products; the head sums differ in order only (a few ulp)."""
    from gsa_b200 import ops

    dI, Lkv, n = 64, 3001, 64
    qI, kI, w, bias = _strided_inputs(1, n, Lkv, HI, seed=11)
    dims = ops.make_dims(4096, 32, 8, 128, HI, dI)
    block = ops.indexer_scores(dims, qI, kI, w, bias, 0.125, q_pos0=Lkv - n, causal=True)
    last = ops.indexer_scores(dims, qI[:, n - 1:], kI, w[:, n - 1:], bias, 0.125, q_pos0=Lkv - 1, causal=True)
    torch.cuda.synchronize()
    a, b = block[0, n - 1].cpu(), last[0, 0].cpu()
    assert torch.allclose(a, b, rtol=0, atol=2e-5), float((a - b).abs().max())


def _layer(HI=8, dtype=torch.bfloat16):
    from gsa_b200 import GSAConfig, GatedSparseAttention

    cfg = GSAConfig(d_model=512, n_heads=8, n_kv_heads=2, d_indexer=64, n_indexer_heads=HI, k_base=192,
                    k_min=64, k_max=384, use_adaptive_k=False, max_position_embeddings=4096)
    torch.manual_seed(0)
    return GatedSparseAttention(cfg).to(DEV).to(dtype).eval()


def _x(B, L, seed, dtype=torch.bfloat16):
    return torch.randn(B, L, 512, generator=torch.Generator().manual_seed(seed)).to(DEV, dtype)


def test_prefill_into_allocated_cache_equals_plain_prefill(cuda_ok):
    m = _layer()
    B, L = 3, 900
    x = _x(B, L, 1)
    with torch.no_grad():
        plain = m(x)[0]
        cache = m.allocate_cache(B, 1024)
        out, c, _ = m(x, past_key_value=cache, use_cache=True)
    torch.cuda.synchronize()
    assert torch.equal(out, plain)
    assert c.store is cache.store and c.capacity == 1024 and c[0].shape == (B, L, 2, 64)
    assert c[0].data_ptr() == cache.store.kv.data_ptr()


def test_decode_appends_in_place_and_branches_copy(cuda_ok):
    m = _layer()
    B, L = 2, 600
    x = _x(B, L + 2, 2)
    with torch.no_grad():
        _, c0, _ = m(x[:, :L], use_cache=True)
        assert c0.capacity > L                                   # the prefill left room
        oa, ca, _ = m(x[:, L:L + 1], past_key_value=c0, use_cache=True)
        assert ca.store is c0.store                              # appended in place
        ka = ca[0][:, L].clone()
        # a second continuation of c0: its slot L is taken, so this one moves to a new store
        ob, cb, _ = m(x[:, L + 1:L + 2], past_key_value=c0, use_cache=True)
        assert cb.store is not c0.store
        assert torch.equal(ca[0][:, L], ka)                      # the first continuation is intact
        assert torch.equal(cb[0][:, :L], c0[0]) and torch.equal(cb.indexer_keys[:, :L], c0.indexer_keys)
        # the same steps on caches that were each copied first give the same outputs
        oa2 = m(x[:, L:L + 1], past_key_value=_copy(c0), use_cache=True)[0]
        ob2 = m(x[:, L + 1:L + 2], past_key_value=_copy(c0), use_cache=True)[0]
    torch.cuda.synchronize()
    assert torch.equal(oa, oa2) and torch.equal(ob, ob2)


def _copy(c):
    from gsa_b200 import GSAKVCache

    return GSAKVCache(c[0].clone(), c[1].clone(), c.indexer_keys.clone())


def test_full_store_grows_with_the_same_results(cuda_ok):
    m = _layer(HI=4)
    B, L, steps = 2, 500, 4
    x = _x(B, L + steps, 3)
    outs = {}
    with torch.no_grad():
        for cap in (L + 1, 4096):
            cache = m.allocate_cache(B, cap)
            out, c, _ = m(x[:, :L], past_key_value=cache, use_cache=True)
            seq = [out]
            for s in range(steps):
                out, c, _ = m(x[:, L + s:L + s + 1], past_key_value=c, use_cache=True)
                seq.append(out)
            outs[cap] = (torch.cat(seq, 1), c)
    torch.cuda.synchronize()
    small, big = outs[L + 1], outs[4096]
    assert small[1].capacity > L + 1 and small[1][0].shape[1] == L + steps
    assert torch.equal(small[0], big[0])
    assert torch.equal(small[1][0], big[1][0]) and torch.equal(small[1].indexer_keys, big[1].indexer_keys)


def test_decode_without_use_cache_leaves_the_cache_unclaimed(cuda_ok):
    """use_cache=False writes the new token into the store's free slot but does not claim it:
    the next continuation of the same cache still appends in place."""
    m = _layer()
    x = _x(1, 301, 4)
    with torch.no_grad():
        _, c0, _ = m(x[:, :300], use_cache=True)
        o1, none, _ = m(x[:, 300:], past_key_value=c0)
        assert none is None and c0.store.filled == 300
        o2, c1, _ = m(x[:, 300:], past_key_value=c0, use_cache=True)
        assert c1.store is c0.store
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


_SPLIT_COUNTS = {
    "ragged": [0, 1, 15, 16, 17, 700, 2049, 4096],
    "mostly_empty": [0, 1, 0, 0, 17, 0, 0, 16],
    "decode64": [0, 4096, 3] + [int(x) for x in torch.randint(0, 4097, (61,),
                                                             generator=torch.Generator().manual_seed(5))],
    "four_rows": [5, 4096, 0, 333],
}


@pytest.mark.parametrize("case", sorted(_SPLIT_COUNTS))
def test_split_sdpa_matches_unsplit_and_reference(cuda_ok, case):
    """Few rows (decode): gsa_sparse_sdpa_strided cuts each row's selected keys over several CTAs
    (8 ranges per row at 4 and 8 rows, 2 at 64) and merges their partial softmax results; against
    the unsplit kernel and fp32 attention.  Rows with 0, 1, 15, 16, 17 and thousands of keys
    (empty and ragged key ranges), mostly empty rows, and 64 decode rows."""
    import ctypes as C

    from gsa_b200 import _lib, ops

    H, Hk, D, Lkv = 32, 8, 128, 6000
    counts = _SPLIT_COUNTS[case]
    B = len(counts)
    g = torch.Generator().manual_seed(21)
    q = torch.randn(B, 1, H, D, generator=g).to(torch.bfloat16).to(DEV)
    store = torch.randn(B, Lkv + 100, 2, Hk, D, generator=g).to(torch.bfloat16).to(DEV)
    kv = store[:, :Lkv]
    k, v = kv[:, :, 0], kv[:, :, 1]
    gate = torch.sigmoid(torch.randn(B, 1, H, D, generator=g)).to(torch.bfloat16).to(DEV)
    sel = torch.zeros(B, 4096, dtype=torch.int32)
    for b, c in enumerate(counts):
        sel[b, :c] = torch.sort(torch.randperm(Lkv, generator=g)[:c]).values.int()
    sel, cnt = sel.to(DEV), torch.tensor(counts, dtype=torch.int32, device=DEV)
    dims = ops.make_dims(H * D, H, Hk, D, 8, 64)
    scale = 1 / math.sqrt(D)
    assert _lib.lib().gsa_sdpa_workspace_size(C.byref(dims), B, 1) > 0      # few rows: a split is offered
    split = ops.sparse_sdpa(dims, q, k, v, sel, cnt, gate, scale)
    whole = torch.empty_like(q)
    _lib.call("gsa_sparse_sdpa_strided", C.byref(dims), 1, B, 1, Lkv, C.c_void_p(q.data_ptr()),
              C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), k.stride(1), k.stride(0),
              C.c_void_p(sel.data_ptr()), sel.stride(0), C.c_void_p(cnt.data_ptr()), C.c_void_p(gate.data_ptr()),
              C.c_void_p(whole.data_ptr()), scale, None, 0, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ops.check_device_error()
    # fp32 reference
    ref = torch.zeros(B, H, D)
    for b, c in enumerate(counts):
        if c == 0:
            continue
        idx = sel[b, :c].long().cpu()
        kk = k[b].float().cpu()[idx].repeat_interleave(H // Hk, dim=1)   # [c, H, D]
        vv = v[b].float().cpu()[idx].repeat_interleave(H // Hk, dim=1)
        p = torch.softmax(torch.einsum("hd,chd->hc", q[b, 0].float().cpu(), kk) * scale, dim=-1)
        ref[b] = torch.einsum("hc,chd->hd", p, vv) * gate[b, 0].float().cpu()
    for out in (split, whole):
        o = out.view(B, H, D).float().cpu()
        for b, c in enumerate(counts):
            if c == 0:
                assert torch.equal(o[b], torch.zeros(H, D))              # no keys: zeros
        err = (o - ref).norm() / ref.norm()
        assert float(err) < 1e-2, float(err)
    assert float((split.float() - whole.float()).abs().max()) < 2e-2


@pytest.mark.parametrize("dtype,HI,adaptive", [(torch.bfloat16, 8, True), (torch.bfloat16, 4, False),
                                               (torch.float32, 8, True)])
def test_native_step_equals_python_step(cuda_ok, dtype, HI, adaptive):
    """The one-call native step (gsa_decode_attend) and the same kernels launched one by one
    from Python give the same outputs, caches and selections bit for bit: prefill into a store,
    then decode steps."""
    from gsa_b200 import GSAConfig, GatedSparseAttention

    cfg = GSAConfig(d_model=512, n_heads=8, n_kv_heads=2, d_indexer=64, n_indexer_heads=HI, k_base=192,
                    k_min=64, k_max=384, use_adaptive_k=adaptive, max_position_embeddings=4096)
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).to(DEV).to(dtype).eval()
    B, L, steps = 3, 700, 3
    x = _x(B, L + steps, 5, dtype)
    res = {}
    with torch.no_grad():
        for native in (True, False):
            m.native_step = native
            out, c, _ = m(x[:, :L], past_key_value=m.allocate_cache(B, L + 64), use_cache=True)
            outs = [out]
            for s in range(steps):
                out, c, _ = m(x[:, L + s:L + s + 1], past_key_value=c, use_cache=True)
                outs.append(out)
            res[native] = (torch.cat(outs, 1), c)
    m.native_step = True
    torch.cuda.synchronize()
    (o1, c1), (o2, c2) = res[True], res[False]
    assert torch.equal(o1, o2)
    assert torch.equal(c1[0], c2[0]) and torch.equal(c1[1], c2[1]) and torch.equal(c1.indexer_keys, c2.indexer_keys)
