"""Cached decode and the analysis outputs.

Decode: with a fixed k (no cross-row variance mean), decoding token L against a GSAKVCache (which
carries the indexer keys, so the new query is scored against every cached key) must give row L
of a prefill over L+1 tokens, and prefilling L tokens with use_cache=True must give the first L
rows.  The selection for those rows is the same; only the o_proj GEMM over one row instead of
L+1 rows may round differently, hence a tolerance.  Several decode steps in a row and batch > 1
are covered, in fp32 and bf16.

Analysis: GatedLightningIndexer.get_indexer_statistics and
AdaptiveTopKSelector.get_selection_statistics against the same statistics computed from the
oracle's scores and k values (gated_indexer.py:157-175, adaptive_topk.py:195-211), and the gates'
last_gate_scores after a layer forward."""

import pytest
import torch

import gsa_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _layer(dtype, adaptive):
    from gsa_b200 import GSAConfig, GatedSparseAttention

    cfg = GSAConfig(d_model=512, n_heads=8, n_kv_heads=2, d_indexer=64, n_indexer_heads=4, k_base=192,
                    k_min=64, k_max=384, use_adaptive_k=adaptive, max_position_embeddings=4096)
    torch.manual_seed(0)
    return GatedSparseAttention(cfg).to(DEV).to(dtype).eval()


def _rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm())


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2)])
def test_cached_decode_matches_prefill(cuda_ok, dtype, tol):
    m = _layer(dtype, adaptive=False)
    B, L, steps = 2, 700, 3
    x = torch.randn(B, L + steps, 512, generator=torch.Generator().manual_seed(1)).to(DEV, dtype)
    with torch.no_grad():
        full = m(x)[0]
        out, cache, _ = m(x[:, :L], use_cache=True)
        assert _rel(out, full[:, :L]) < tol
        assert cache.indexer_keys is not None and cache[0].shape[1] == L
        for s in range(steps):
            out, cache, _ = m(x[:, L + s:L + s + 1], past_key_value=cache, use_cache=True)
            assert cache[0].shape[1] == L + s + 1
            err = _rel(out[:, 0], full[:, L + s])
            assert err < tol, (s, err)
    torch.cuda.synchronize()


def test_cached_decode_keys_equal_prefill_keys(cuda_ok):
    """The cache after prefill + decode holds exactly the K, V and k^I a longer prefill produces."""
    m = _layer(torch.bfloat16, adaptive=True)
    B, L = 1, 513
    x = torch.randn(B, L + 1, 512, generator=torch.Generator().manual_seed(2)).to(DEV, torch.bfloat16)
    with torch.no_grad():
        _, c_full, _ = m(x, use_cache=True)
        _, c, _ = m(x[:, :L], use_cache=True)
        _, c, _ = m(x[:, L:], past_key_value=c, use_cache=True)
    torch.cuda.synchronize()
    assert torch.equal(c[0], c_full[0]) and torch.equal(c[1], c_full[1])
    assert torch.equal(c.indexer_keys, c_full.indexer_keys)


def test_analysis_statistics_match_oracle(cuda_ok):
    from gsa_b200 import AdaptiveTopKSelector

    m = _layer(torch.float32, adaptive=True)
    ix = m.indexer
    B, L = 1, 300
    h = torch.randn(B, L, 512, generator=torch.Generator().manual_seed(3)).to(DEV)
    stats = ix.get_indexer_statistics(h)
    with torch.no_grad():
        q_idx = ix.q_proj(h).view(B, L, 4, 64).cpu()
        k_idx = ix.k_proj(h).cpu()
        w = torch.sigmoid(ix.weight_proj(h)).cpu()
    ref = O.indexer_scores_from_proj(q_idx, k_idx, w, ix.bias.detach().cpu(), "sigmoid", q_offset=0)
    valid = ref[ref != float("-inf")]
    for key, val in (("mean", valid.mean()), ("std", valid.std()), ("min", valid.min()), ("max", valid.max())):
        assert abs(stats[key] - float(val)) <= 1e-4 * max(1.0, abs(float(val))), key
    assert abs(stats["sparsity"] - float((valid < 0.1).float().mean())) < 1e-3
    assert stats["head_weights"] == torch.sigmoid(ix.weight_proj.bias).tolist()

    sel = AdaptiveTopKSelector(k_base=96, k_min=32, k_max=160, temperature=1.0)
    s = ref.to(DEV)
    got = sel.get_selection_statistics(s)
    var, cnt = O.row_variance(ref)
    kv = O.adaptive_k(var, cnt, var.mean(), 96, 32, 160, 1.0)
    _, _, k_ours = sel(s, L, L, return_k_values=True)
    assert torch.equal(k_ours.cpu(), kv.long())          # the k_t themselves: exact
    k_eff = min(160, L)
    kf = kv.float()                                      # the statistics are taken in fp32
    assert abs(got["k_mean"] - float(kf.mean())) <= 1e-6 * float(kf.mean())
    assert abs(got["k_std"] - float(kf.std())) <= 1e-5 * float(kf.std())
    assert got["k_min"] == int(kv.min()) and got["k_max"] == int(kv.max())
    assert abs(got["coverage"] - float(kv.sum()) / (B * L * k_eff)) < 1e-6


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_batch_rows_equal_separate_calls(cuda_ok, dtype):
    """A B = 3 forward equals three B = 1 forwards (fixed k: the adaptive k's variance mean spans
    every row of a call, so it would differ by design)."""
    m = _layer(dtype, adaptive=False)
    x = torch.randn(3, 1100, 512, generator=torch.Generator().manual_seed(4)).to(DEV, dtype)
    with torch.no_grad():
        both = m(x)[0]
        each = torch.cat([m(x[b:b + 1])[0] for b in range(3)])
    torch.cuda.synchronize()
    # the same kernels on the same rows; only the GEMMs' blocking may differ with the row count
    assert _rel(both, each) < (1e-5 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2)])
def test_gate_scores_after_layer_forward(cuda_ok, dtype, tol):
    """After an eval-mode layer forward the gates hold their activations for analysis
    (value_gate.py:109-110, output_gate.py:122-123): act(h W^T + b) of the layer's input, per
    KV-head (G2) and per head (G1) element; get_gate_statistics reads them."""
    import torch.nn.functional as F

    m = _layer(dtype, adaptive=True)
    x = torch.randn(2, 300, 512, generator=torch.Generator().manual_seed(6)).to(DEV, dtype)
    with torch.no_grad():
        m(x)
        vg, og = m.value_gate, m.output_gate
        ref_v = torch.sigmoid(F.linear(x, vg.gate_proj.weight, vg.gate_proj.bias)).view(2, 300, 2, 64)
        ref_o = torch.sigmoid(F.linear(x, og.gate_proj.weight, og.gate_proj.bias)).view(2, 300, 8, 64)
        got_v, got_o = vg.last_gate_scores, og.last_gate_scores
    torch.cuda.synchronize()
    assert got_v.shape == ref_v.shape and got_o.shape == ref_o.shape and got_v.dtype == dtype
    assert float((got_v.float() - ref_v.float()).abs().max()) < tol
    assert float((got_o.float() - ref_o.float()).abs().max()) < tol
    stats = vg.get_gate_statistics()
    assert abs(stats["mean"] - float(ref_v.float().mean())) < tol
