"""The tensor-core indexer (bf16, d_I = 64, H_I in {4, 8}) and the chunked indexer + top-k path
against the CPU oracle, at shapes with ragged edges: key counts that are not multiples of the
128-key tile, partial query blocks, query offsets (a later chunk or a query shard), batch > 1."""

import math

import numpy as np
import pytest
import torch

import gsa_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(B, Lq, Lkv, HI, dI=64, seed=0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    qI = (torch.randn(B, Lq, HI * dI, generator=g) * 1.3).to(dtype)
    kI = (torch.randn(B, Lkv, dI, generator=g) * 1.4).to(dtype)
    w = torch.sigmoid(torch.randn(B, Lq, HI, generator=g) * 0.3).to(dtype).float()
    bias = torch.randn(HI, generator=g) * 0.1
    return qI, kI, w, bias


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


@pytest.mark.parametrize("B,Lq,Lkv,HI,q_pos0,causal", [
    (1, 384, 384, 8, 0, True),
    (2, 700, 700, 8, 0, True),
    (1, 257, 1300, 8, 1043, True),      # a later query chunk: offset-causal
    (1, 130, 1000, 4, 0, False),        # non-causal (decode-like), H_I = 4
    (1, 64, 4097, 8, 4033, True),
])
def test_tensor_core_indexer_matches_oracle(cuda_ok, B, Lq, Lkv, HI, q_pos0, causal):
    from gsa_b200 import ops

    dI = 64
    qI, kI, w, bias = _inputs(B, Lq, Lkv, HI)
    dims = ops.make_dims(4096, 32, 8, 128, HI, dI)
    stats = torch.zeros(B * Lq, 3, device=DEV, dtype=torch.float64)
    ours = ops.indexer_scores(dims, qI.to(DEV), kI.to(DEV), w.to(DEV), bias.to(DEV), 1 / math.sqrt(dI),
                              q_pos0=q_pos0, causal=causal, row_stats=stats)
    torch.cuda.synchronize()
    ops.check_device_error()
    ref = _oracle_scores(qI, kI, w, bias, HI, dI, q_pos0, causal)
    ours = ours.cpu()
    inf = torch.isinf(ref)
    assert torch.equal(torch.isinf(ours), inf)
    err = (ours[~inf] - ref[~inf]).abs() / ref[~inf].abs()
    assert float(err.max()) < 2e-2, float(err.max())
    assert float(err.mean()) < 2e-3
    # row statistics: sum, sum of squares and count of unmasked entries
    valid = ~inf.view(B * Lq, Lkv)
    r = ref.view(B * Lq, Lkv).double()
    cnt = valid.sum(-1).double()
    s1 = torch.where(valid, r, torch.zeros_like(r)).sum(-1)
    st = stats.cpu()
    assert torch.equal(st[:, 2], cnt)
    assert torch.allclose(st[:, 0], s1, rtol=2e-3, atol=1e-3)


@pytest.mark.parametrize("HI", [8, 4])
def test_chunked_select_equals_materialised_select(cuda_ok, HI):
    """gsa_indexer_select (chunked, no full score matrix) keeps the same candidates as top-k run
    on the materialised scores of the same kernel."""
    from gsa_b200 import ops

    B, L, dI, k_eff = 1, 1500, 64, 200
    qI, kI, w, bias = _inputs(B, L, L, HI, seed=3)
    qI, kI, w, bias = qI.to(DEV), kI.to(DEV), w.to(DEV), bias.to(DEV)
    dims = ops.make_dims(4096, 32, 8, 128, HI, dI)
    shift = 0.5 * w.view(B * L, HI).sum(-1)
    ci, cs, cc, stats = ops.indexer_select(dims, qI, kI, w, bias, 1 / math.sqrt(dI), shift, k_eff,
                                           q_pos0=0, causal=True, chunk_rows=333)
    full = ops.indexer_scores(dims, qI, kI, w, bias, 1 / math.sqrt(dI), q_pos0=0, causal=True)
    ri, rs, rc = ops.topk_candidates(full.view(B * L, L), k_eff, Lq=L, q_pos0=0, causal=True)
    torch.cuda.synchronize()
    ops.check_device_error()
    assert torch.equal(cc, rc)
    assert torch.equal(ci, ri)
    valid = torch.arange(k_eff, device=DEV).view(1, -1) < cc.view(-1, 1)
    assert torch.equal(cs[valid], rs[valid])
    assert torch.equal(cc.cpu(), torch.clamp(torch.arange(L) + 1, max=k_eff).int())
    # the candidates of every row are its k_eff best scores, in ascending column order
    f = full.view(L, L).cpu()
    for r in [0, 5, 199, 200, 777, L - 1]:
        n = int(cc[r])
        idx = ci[r, :n].cpu().long()
        assert bool((idx[1:] > idx[:-1]).all())
        assert int(idx.max()) <= r
        row = f[r, :r + 1]
        kept = torch.zeros(r + 1, dtype=torch.bool)
        kept[idx] = True
        if n < r + 1:
            assert float(row[kept].min()) >= float(row[~kept].max())


def test_topk_ties_take_lower_columns(cuda_ok):
    """Equal scores at the cut are taken lowest column first."""
    from gsa_b200 import ops  # noqa: F811

    L = 5000
    s = torch.full((3, L), 1.0)
    s[0, ::7] = 2.0                       # 715 values of 2, the rest ties at 1
    s[1] = torch.arange(L).float() % 10   # many ties per level
    s[2, :100] = float("-inf")            # masked prefix
    k = 1000
    idx, sc, cnt = ops.topk_candidates(s.to(DEV), k)
    torch.cuda.synchronize()
    for r in range(3):
        ours = np.sort(idx[r, :int(cnt[r])].cpu().numpy())
        ref = O.topk_sets_stable(s[r:r + 1], torch.tensor([k]))[0]
        assert np.array_equal(ours, ref), r


@pytest.mark.parametrize("n,k", [(20000, 4096), (3000, 512), (131072, 4096), (700, 4096)])
def test_bounded_range_selection_equals_radix(cuda_ok, n, k):
    """The two-pass bounded-range selection keeps exactly the radix select's candidates,
    including rows that are all ties or too concentrated for the compact buffer."""
    from gsa_b200 import ops

    g = torch.Generator().manual_seed(n)
    R = 6
    c = torch.rand(R, generator=g) * 3 + 0.5
    s = torch.sigmoid(torch.randn(R, n, generator=g) * 2) * (2 * c.view(-1, 1))
    s[1] = c[1]                                  # one value: every column ties
    s[2] = torch.round(s[2] * 8) / 8             # heavy ties at few levels
    s[3, n // 2:] = float("-inf")                # masked tail
    s[4] = c[4] * (1 + 1e-6 * torch.rand(n, generator=g))   # all in one bin: overflow fallback
    s = s.contiguous()
    sd = s.to(DEV)
    ri, rs, rc = ops.topk_candidates(sd, k)
    # row statistics relative to the centre, as the indexer produces them
    fin = torch.isfinite(s)
    y = torch.where(fin, s.double() - c.double().view(-1, 1), torch.zeros_like(s, dtype=torch.float64))
    stats = torch.stack([y.sum(-1), (y * y).sum(-1), fin.sum(-1).double()], -1).to(DEV)
    for st in (None, stats):
        bi, bs, bc = ops.topk_candidates(sd, k, row_center=c.to(DEV), row_stats=st)
        torch.cuda.synchronize()
        ops.check_device_error()
        assert torch.equal(rc, bc)
        valid = torch.arange(k, device=DEV).view(1, -1) < rc.view(-1, 1)
        assert torch.equal(ri[valid], bi[valid])
        assert torch.equal(rs[valid], bs[valid])
        for r in range(R):
            ref = O.topk_sets_stable(s[r:r + 1], torch.tensor([k]))[0]
            assert np.array_equal(np.sort(bi[r, :int(bc[r])].cpu().numpy()), ref), r
