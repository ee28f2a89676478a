"""The decoder layer and causal LM on the B200 kernels (gsa/models/gsa_llama.py) against the
reference's own outputs (golden fixtures) and the oracle:

* the fused residual-add + RMSNorm and silu-product kernels against the reference's torch
  formulas: within one unit in the last place of the dtype;
* the two-layer GSALlamaForCausalLM fixture: fp32 logits and every layer's output close to the
  reference's; bf16 logits no further from the exact (fp32) model than the reference's bf16 model
  is (its bf16 indexer scores tie at the k_t boundary, which torch.topk breaks arbitrarily);
* greedy generate with the in-place caches picks the argmax of a full forward at every step;
* a loss backward through the model reaches every trainable parameter but the indexer's."""

import pytest
import torch
import torch.nn.functional as F

from conftest import load_golden
import gsa_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ulp_close(a, b, dtype):
    a, b = a.float().cpu(), b.float().cpu()
    if dtype == torch.float32:
        return bool(torch.allclose(a, b, rtol=2e-6, atol=1e-7))
    eps = 2.0 ** -7  # one bf16 unit in the last place, relative
    return bool(((a - b).abs() <= eps * b.abs() + 1e-30).all())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_norm_and_swiglu_kernels(cuda_ok, dtype):
    from gsa_b200 import ops

    g = torch.Generator().manual_seed(3)
    x = (torch.randn(300, 1024, generator=g) * 2).to(dtype)
    a = torch.randn(300, 1024, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(1024, generator=g)).to(dtype)
    h, y = ops.add_rmsnorm(x.to(DEV), a.to(DEV), w.to(DEV), 1e-5)
    _, y0 = ops.add_rmsnorm(x.to(DEV), None, w.to(DEV), 1e-5, want_sum=False)
    torch.cuda.synchronize()
    ref_h = x + a
    assert torch.equal(h.cpu(), ref_h)
    assert _ulp_close(y, O.rms_norm(ref_h, w, 1e-5), dtype)
    assert _ulp_close(y0, O.rms_norm(x, w, 1e-5), dtype)
    gu = (torch.randn(257, 2 * 700, generator=g) * 3).to(dtype)
    z = ops.silu_mul(gu.to(DEV))
    torch.cuda.synchronize()
    assert _ulp_close(z, F.silu(gu[:, :700]) * gu[:, 700:], dtype)


def _model(name):
    from gsa_b200 import GSAConfig, GSALlamaForCausalLM

    g, meta = load_golden(name)
    cfg = GSAConfig(**meta["config"])
    torch.manual_seed(int(meta["weight_seed"]))
    m = GSALlamaForCausalLM(cfg).eval().to(getattr(torch, meta["dtype"]))
    return g, cfg, m


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm())


def test_causal_lm_fp32_matches_reference(cuda_ok):
    """Every row keeps all its keys: the model agrees with the reference to fp32 rounding."""
    g, cfg, m = _model("model2dense_fp32_b2_l96")
    m = m.to(DEV)
    with torch.no_grad():
        out = m(g["input_ids"].long().to(DEV), output_hidden_states=True)
    torch.cuda.synchronize()
    # hidden_states: the embedding, each layer's output but the last, then the final normed state
    # (gsa_llama.py:207-230)
    for i in range(cfg.n_layers - 1):
        assert _rel(out.hidden_states[i + 1], g[f"layer{i}_out"]) < 1e-4, i
    assert _rel(out.logits, g["logits"]) < 1e-4


def test_causal_lm_fp32_sparse_matches_reference(cuda_ok):
    """Sparse selection (k 8..48 of up to 96 keys; distinct tokens, so no exact score ties): the
    model agrees with the reference to fp32 rounding, row by row."""
    g, cfg, m = _model("model2_fp32_b2_l96")
    m = m.to(DEV)
    with torch.no_grad():
        logits = m(g["input_ids"].long().to(DEV)).logits.double().cpu()
    torch.cuda.synchronize()
    ref = g["logits"].double()
    row_err = (logits - ref).norm(dim=-1) / ref.norm(dim=-1)
    assert float(row_err.max()) < 1e-4, row_err


def test_causal_lm_bf16_within_the_reference_bf16_error(cuda_ok):
    g, cfg, m = _model("model2_bf16_b2_l96")
    ids = g["input_ids"].long()
    W32 = {k: v.float() for k, v in m.state_dict().items()}
    rope = m.model.layers[0].self_attn.rotary_emb
    exact = O.causal_lm_forward(W32, O.OracleConfig.from_config(cfg), cfg.n_layers, cfg.norm_eps, ids,
                                None, None, chunk=32)["logits"]
    m = m.to(DEV)
    with torch.no_grad():
        ours = m(ids.to(DEV)).logits
    torch.cuda.synchronize()
    err, ref_err = _rel(ours, exact), _rel(g["logits"], exact)
    assert err <= max(3e-2, ref_err), (err, ref_err)


def test_greedy_generate_follows_full_forward_argmax(cuda_ok):
    from gsa_b200 import GSAConfig, GSALlamaForCausalLM

    # fixed k: a cached step's selection then equals the full forward's for the same row
    cfg = GSAConfig(d_model=256, n_heads=4, n_kv_heads=2, d_indexer=32, n_indexer_heads=4, k_base=24,
                    k_min=8, k_max=48, use_adaptive_k=False, n_layers=2, d_ffn=512, vocab_size=384,
                    max_position_embeddings=512)
    torch.manual_seed(0)
    m = GSALlamaForCausalLM(cfg).eval().to(DEV)
    ids = torch.randint(0, 384, (2, 40), generator=torch.Generator().manual_seed(1)).to(DEV)
    new = 6
    with torch.no_grad():
        seq = m.generate(ids, max_new_tokens=new, do_sample=False)
        full = m(seq[:, :-1]).logits
    torch.cuda.synchronize()
    assert seq.shape == (2, 40 + new)
    for t in range(40, 40 + new):
        row = full[:, t - 1]
        picked = row.gather(1, seq[:, t:t + 1])
        # the picked token is a maximum of the full forward's logits (up to fp32 rounding)
        assert bool((picked >= row.max(-1, keepdim=True).values - 1e-4).all()), t


def test_loss_backward_reaches_the_trainable_parameters(cuda_ok):
    from gsa_b200 import GSAConfig, GSALlamaForCausalLM

    cfg = GSAConfig(d_model=256, n_heads=4, n_kv_heads=2, d_indexer=32, n_indexer_heads=4, k_base=24,
                    k_min=8, k_max=48, n_layers=2, d_ffn=512, vocab_size=384, max_position_embeddings=512)
    torch.manual_seed(0)
    m = GSALlamaForCausalLM(cfg).to(DEV).train()
    ids = torch.randint(0, 384, (2, 64), generator=torch.Generator().manual_seed(2)).to(DEV)
    out = m(ids, labels=ids)
    out.loss.backward()
    torch.cuda.synchronize()
    assert bool(torch.isfinite(out.loss))
    for name, p in m.named_parameters():
        if ".indexer." in name:
            assert p.grad is None, name
        else:
            assert p.grad is not None and bool(torch.isfinite(p.grad).all()), name
            assert float(p.grad.abs().sum()) > 0, name
