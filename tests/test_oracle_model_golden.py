"""Pins the oracle's restatement of the reference's decoder layer and causal LM
(gsa/models/gsa_llama.py: RMSNorm, SwiGLU MLP, GSADecoderLayer, GSALlamaForCausalLM) to the
reference's own outputs (tests/golden/make_golden.py, two-layer model, fp32 and bf16): weights
regenerate from the seed in our module classes, and every layer's output and the logits agree bit
for bit."""

import pytest
import torch

from conftest import load_golden
import gsa_oracle as O


def _model(meta):
    from gsa_b200 import GSAConfig, GSALlamaForCausalLM

    cfg = GSAConfig(**meta["config"])
    torch.manual_seed(int(meta["weight_seed"]))
    m = GSALlamaForCausalLM(cfg).eval().to(getattr(torch, meta["dtype"]))
    return cfg, m


@pytest.mark.parametrize("name", ["model2_fp32_b2_l96", "model2_bf16_b2_l96", "model2dense_fp32_b2_l96"])
def test_causal_lm_oracle_matches_reference(name):
    g, meta = load_golden(name)
    cfg, m = _model(meta)
    sd = m.state_dict()
    for k, (s, ss, first) in meta["param_checksums"].items():
        t = sd[k].double()
        assert abs(float(t.sum()) - s) <= 1e-9 * max(1.0, abs(s)), k
        assert [float(v) for v in t.flatten()[:4]] == first, k
    W = dict(sd)
    ids = g["input_ids"].long()
    rope = m.model.layers[0].self_attn.rotary_emb
    res = O.causal_lm_forward(W, O.OracleConfig.from_config(cfg), cfg.n_layers, cfg.norm_eps, ids,
                              rope.cos_cached, rope.sin_cached, chunk=32, keep_layers=True)
    for i in range(cfg.n_layers):
        for part in ("normed", "attn", "out"):
            key = f"layer{i}_{part}"
            assert torch.equal(res[key], g[key]), key
    assert torch.equal(res["logits"], g["logits"])
