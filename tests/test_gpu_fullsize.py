"""The 4096-wide layer (d_model 4096, 32/8 heads of 128, 8 indexer heads of 64, k_base 2048, bf16) at
its full workload sizes, checked through properties that do not need a full-size oracle:

  * "c4": one 131072-token sequence, k in [256, 4096] (the headline workload);
  * "c2": two 8192-token sequences, k in [256, 4096] (the README quickstart batch: the adaptive-k
    variance mean spans both sequences, adaptive_topk.py:93-96);
  * "c3": one 32768-token sequence, k clipped to [512, 4096].

Checked for each:

* every row's selection: ascending, unique, causal (keys <= the row's position), exactly k_t keys,
  and k_t = clamp(k_base * (0.5 + 1 / (1 + v/mean)), k_min, k_max) limited by the row's key count
  (adaptive_topk.py:96-136) -- its bounds are checked for every row;
* sampled rows across each sequence against a torch fp32 recomputation from the layer's own
  projections: every kept key's indexer score (gated_indexer.py:114-153) is at least every dropped
  key's within the tanh.approx error of the bf16 indexer (2e-3 of the score range), and the
  attention output (gated_sparse_attention.py:256-290, G1 gate) matches within 2e-2;
* c2 and c3 (whose score matrices a GPU recomputation can hold chunk by chunk): every row's k_t
  against the variance of its fp32-recomputed scores, with the mean over all rows of the batch, in
  the reference's bf16 arithmetic (at most one key apart where the two variances round apart)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"

SHAPES = {"c4": (1, 131072, 256, 4096), "c2": (2, 8192, 256, 4096), "c3": (1, 32768, 512, 4096)}


def _rows(L):
    return sorted({0, 1, 255, 256, 511, 512, 4095, 4096, L // 4 + 1, L // 2, (3 * L) // 4 + 7, L - 1} & set(range(L)))


@pytest.fixture(scope="module", params=["c2", "c3", "c4"])
def shape(request):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gsa_b200 import GSAConfig, GatedSparseAttention

    name = request.param
    B, L, k_min, k_max = SHAPES[name]
    cfg = GSAConfig(d_model=4096, n_heads=32, n_kv_heads=8, d_indexer=64, n_indexer_heads=8, k_base=2048,
                    k_min=k_min, k_max=k_max, max_position_embeddings=max(L, 131072))
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).eval().to(torch.bfloat16).to(DEV)
    x = torch.randn(B, L, 4096, generator=torch.Generator().manual_seed(1)).to(DEV, torch.bfloat16)
    cap = {}
    with torch.no_grad():
        m._forward_impl(x, None, None, False, False, capture=cap)
    torch.cuda.synchronize()
    from gsa_b200 import ops
    ops.check_device_error()
    yield name, B, L, cfg, m, cap
    del cap, m, x
    torch.cuda.empty_cache()


def test_every_row_selection_is_ascending_causal_and_k_t_long(shape):
    name, B, L, cfg, m, cap = shape
    sel, cnt, kt = cap["sel"], cap["cnt"].long(), cap["k_t"].long()
    R, ld = sel.shape
    assert R == B * L
    pos = torch.arange(R, device=DEV) % L
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


def _scores_fp32(cap, cfg, b, L, t0, t1):
    """fp32 indexer scores of rows [t0, t1) of sequence b against every key, -inf above the diagonal."""
    HI, dI = cfg.n_indexer_heads, cfg.d_indexer
    q = cap["qI"][b, t0:t1].float().view(t1 - t0, HI, dI)
    keys = cap["kI"][b].float()
    w = cap["w"].view(-1, L, HI)[b, t0:t1]
    bias = cap["bias"].detach().float()
    z = torch.einsum("thd,sd->tsh", q, keys) / math.sqrt(dI) + bias
    s = (torch.sigmoid(z) * w[:, None, :]).sum(-1)                           # [t1-t0, L]
    t = torch.arange(t0, t1, device=DEV).view(-1, 1)
    return s.masked_fill(torch.arange(L, device=DEV).view(1, -1) > t, float("-inf"))


def test_sampled_rows_keep_their_best_keys(shape):
    name, B, L, cfg, m, cap = shape
    w = cap["w"].view(B, L, cfg.n_indexer_heads)
    for b in range(B):
        for t in _rows(L):
            s = _scores_fp32(cap, cfg, b, L, t, t + 1)[0, :t + 1]
            r = b * L + t
            c = int(cap["cnt"][r])
            kept = cap["sel"][r, :c].long()
            mask = torch.ones(t + 1, dtype=torch.bool, device=DEV)
            mask[kept] = False
            tol = 2e-3 * float(w[b, t].sum())
            if bool(mask.any()):
                assert float(s[kept].min()) >= float(s[mask].max()) - tol, (name, b, t)


def test_sampled_rows_attention(shape):
    name, B, L, cfg, m, cap = shape
    H, Hk, D = cfg.n_heads, cfg.n_kv_heads, cfg.d_head
    q, k, v, attn = cap["q"], cap["k"], cap["v"], cap["attn"]
    gate = cap["gate"].view(B, L, H, D)
    for b in range(B):
        for t in _rows(L):
            r = b * L + t
            c = int(cap["cnt"][r])
            idx = cap["sel"][r, :c].long()
            kk = k[b, idx].float().repeat_interleave(H // Hk, dim=1)   # [c, H, D]
            vv = v[b, idx].float().repeat_interleave(H // Hk, dim=1)
            p = torch.softmax(torch.einsum("hd,chd->hc", q[b, t].float(), kk) / math.sqrt(D), dim=-1)
            ref = torch.einsum("hc,chd->hd", p, vv) * gate[b, t].float()
            err = float((attn[b, t].float() - ref).norm() / ref.norm())
            assert err < 2e-2, (name, b, t, err)


def test_every_row_k_t_from_recomputed_variance(shape):
    """Every row's adaptive k.  (1) The layer's k_t is the reference's bf16 formula (the oracle's
    adaptive_k, adaptive_topk.py:96-136) applied to the layer's own row variances and their mean
    over every row of the batch (:96): exactly.  (2) Those variances are the unbiased variance of
    the row's fp32-recomputed scores with masked entries counted as 0 (:84-93), to one bf16 unit
    in the last place (the bf16 indexer's tanh.approx moves a score by ~1e-3 of its range)."""
    import gsa_oracle as O

    name, B, L, cfg, m, cap = shape
    var_ours = cap["var"].cpu().view(B, L).to(torch.bfloat16)
    total = cap["var_total"].cpu()
    mean = torch.tensor(float(torch.tensor(float(total[0]), dtype=torch.float32) /
                              torch.tensor(float(total[1]), dtype=torch.float32))).to(torch.bfloat16)
    assert int(total[1]) == B * L
    valid = (torch.arange(L, dtype=torch.float32) + 1).expand(B, L)
    k_formula = O.adaptive_k(var_ours, valid, mean, cfg.k_base, cfg.k_min, cfg.k_max, 1.0)
    ours = cap["k_t"].long().cpu().view(B, L)
    assert torch.equal(ours, k_formula)
    if name == "c4":
        return  # a recomputation of 131072 x 131072 scores is left to the sampled rows
    var = torch.empty(B, L, dtype=torch.float64)
    for b in range(B):
        for t0 in range(0, L, 1024):
            s = _scores_fp32(cap, cfg, b, L, t0, min(L, t0 + 1024)).double()
            s = torch.where(torch.isinf(s), torch.zeros_like(s), s)
            var[b, t0:t0 + s.shape[0]] = s.var(dim=-1).cpu()
    var_b = var.to(torch.bfloat16)
    ulp = (var_b.float().abs() * 2.0 ** -7).clamp_min(1e-30)
    gap = (var_ours.float() - var_b.float()).abs()
    n_diff = int((gap > 0).sum())
    print(f"{name}: row variances equal to the fp32 recomputation in {B * L - n_diff} of {B * L} rows")
    assert bool((gap <= ulp * 1.01).all()), float((gap / ulp).max())
    rel_mean = abs(float(mean) - float(var_b.float().mean())) / float(var_b.float().mean())
    assert rel_mean <= 2.0 ** -7, rel_mean
    if B > 1:
        # the mean spans the batch: k_t with one sequence's own mean differs in some rows
        for b in range(B):
            own = var_ours[b].float().mean().to(torch.bfloat16)
            k_own = O.adaptive_k(var_ours[b:b + 1], valid[b:b + 1], own, cfg.k_base, cfg.k_min, cfg.k_max, 1.0)[0]
            print(f"{name}: sequence {b}: own mean {float(own):.6g} vs batch mean {float(mean):.6g}; "
                  f"{int((k_own != ours[b]).sum())} rows would take another k_t")


def test_repeated_forwards_are_bit_identical(shape):
    """Three more forwards of the same input give the first forward's selection, k_t and output bit
    for bit: the indexer's per-row statistics are summed in a fixed order (per key-range partials,
    not fp64 atomics), so no row's variance can round differently from run to run."""
    from gsa_b200 import ops

    name, B, L, cfg, m, cap = shape
    x = torch.randn(B, L, 4096, generator=torch.Generator().manual_seed(1)).to(DEV, torch.bfloat16)
    for _ in range(3):
        c2 = {}
        with torch.no_grad():
            m._forward_impl(x, None, None, False, False, capture=c2)
        torch.cuda.synchronize()
        ops.check_device_error()
        assert torch.equal(c2["k_t"], cap["k_t"]), name
        assert torch.equal(c2["cnt"], cap["cnt"]), name
        assert torch.equal(c2["attn"], cap["attn"]), name
        del c2
