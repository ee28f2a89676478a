"""The layer at the headline size (one 131072-token sequence, d_model 4096, 32/8 heads of 128,
8 indexer heads of 64, k_base 2048 in [256, 4096], bf16), checked through properties that do not
need a full-size oracle:

* every row's selection: ascending, unique, causal (keys <= the row's position), exactly k_t keys,
  and k_t = clamp(k_base * (0.5 + 1 / (1 + v/mean)), k_min, k_max) limited by the row's key count
  (adaptive_topk.py:96-136) -- its bounds are checked for every row;
* sampled rows across the sequence against a torch fp32 recomputation from the layer's own
  projections: every kept key's indexer score (gated_indexer.py:114-153) is at least every dropped
  key's within the tanh.approx error of the bf16 indexer (2e-3 of the score range), and the
  attention output (gated_sparse_attention.py:256-290, G1 gate) matches within 2e-2."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
L = 131072


@pytest.fixture(scope="module")
def c4():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gsa_b200 import GSAConfig, GatedSparseAttention

    cfg = GSAConfig(d_model=4096, n_heads=32, n_kv_heads=8, d_indexer=64, n_indexer_heads=8, k_base=2048,
                    k_min=256, k_max=4096, max_position_embeddings=L)
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).eval().to(torch.bfloat16).to(DEV)
    x = torch.randn(1, L, 4096, generator=torch.Generator().manual_seed(1)).to(DEV, torch.bfloat16)
    cap = {}
    with torch.no_grad():
        m._forward_impl(x, None, None, False, False, capture=cap)
    torch.cuda.synchronize()
    return cfg, m, cap


def test_every_row_selection_is_ascending_causal_and_k_t_long(c4):
    cfg, m, cap = c4
    sel, cnt, kt = cap["sel"], cap["cnt"].long(), cap["k_t"].long()
    R, ld = sel.shape
    pos = torch.arange(R, device=DEV)
    n = pos + 1
    assert torch.equal(cnt, torch.minimum(kt, n))
    lo = torch.minimum(torch.full_like(n, cfg.k_min), n)
    hi = torch.minimum(torch.full_like(n, cfg.k_max), n)
    assert bool(((kt >= lo) & (kt <= hi)).all())
    for r0 in range(0, R, 16384):  # in row blocks, to bound the temporaries
        s = sel[r0:r0 + 16384].long()
        c = cnt[r0:r0 + 16384].view(-1, 1)
        j = torch.arange(ld, device=DEV).view(1, -1)
        valid = j < c
        steps = valid[:, 1:] & (s[:, 1:] <= s[:, :-1])
        assert not bool(steps.any()), r0                                   # strictly ascending
        assert not bool((valid & ((s < 0) | (s > pos[r0:r0 + 16384].view(-1, 1)))).any()), r0   # causal


ROWS = [0, 1, 255, 256, 4095, 4096, 30001, 65536, 98765, 131071]


def test_sampled_rows_keep_their_best_keys(c4):
    cfg, m, cap = c4
    HI, dI = cfg.n_indexer_heads, cfg.d_indexer
    qI, kI = cap["qI"][0], cap["kI"][0].float()
    w = cap["w"].view(L, HI)
    bias = cap["bias"].detach().float()
    scale = 1.0 / math.sqrt(dI)
    for t in ROWS:
        q = qI[t].float().view(HI, dI)
        keys = kI[:t + 1]
        s = (torch.sigmoid(keys @ q.t() * scale + bias) * w[t]).sum(-1)    # [t+1], fp32
        c = int(cap["cnt"][t])
        kept = cap["sel"][t, :c].long()
        mask = torch.ones(t + 1, dtype=torch.bool, device=DEV)
        mask[kept] = False
        tol = 2e-3 * float(w[t].sum())
        if bool(mask.any()):
            assert float(s[kept].min()) >= float(s[mask].max()) - tol, t


def test_sampled_rows_attention(c4):
    cfg, m, cap = c4
    H, Hk, D = cfg.n_heads, cfg.n_kv_heads, cfg.d_head
    q, k, v, gate, attn = cap["q"][0], cap["k"][0], cap["v"][0], cap["gate"], cap["attn"][0]
    gate = gate.view(L, H, D)
    for t in ROWS:
        c = int(cap["cnt"][t])
        idx = cap["sel"][t, :c].long()
        kk = k[idx].float().repeat_interleave(H // Hk, dim=1)   # [c, H, D]
        vv = v[idx].float().repeat_interleave(H // Hk, dim=1)
        p = torch.softmax(torch.einsum("hd,chd->hc", q[t].float(), kk) / math.sqrt(D), dim=-1)
        ref = torch.einsum("hc,chd->hd", p, vv) * gate[t].float()
        err = float((attn[t].float() - ref).norm() / ref.norm())
        assert err < 2e-2, (t, err)
