"""Backward of the layer (training): gradients of every differentiable parameter and of the input
against torch autograd through the oracle's restatement of the reference's forward
(gated_sparse_attention.py:175-232 with value_gate.py, rope.py, output_gate.py), on the same
selection (the selection has no gradient: adaptive_topk.py:177 takes torch.topk indices).  The
indexer's parameters get no gradient, as in the reference.  fp32 (tight) and bf16 (against the
fp32 gradient), head dims 64 and 128, adaptive and fixed k."""

import math

import pytest
import torch
import torch.nn.functional as F

import gsa_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _layer(d_model, n_heads, n_kv, HI, dtype, adaptive=True, gate_act="sigmoid"):
    from gsa_b200 import GSAConfig, GatedSparseAttention

    cfg = GSAConfig(d_model=d_model, n_heads=n_heads, n_kv_heads=n_kv, d_indexer=64, n_indexer_heads=HI,
                    k_base=96, k_min=32, k_max=192, use_adaptive_k=adaptive, max_position_embeddings=2048)
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).to(DEV).to(dtype).train()
    # the layer builds its gates with their default activation (as the reference does); other
    # activations are set on the gate modules
    m.value_gate.activation = m.output_gate.activation = gate_act
    return m, cfg


def _reference_grads(m, cfg, x, sel, cnt, R):
    """fp32 autograd through the oracle forward with the given selection."""
    W = {k: v.detach().float().cpu().clone().requires_grad_(True) for k, v in m.state_dict().items()
         if not k.startswith("rotary_emb")}
    xr = x.detach().float().cpu().clone().requires_grad_(True)
    B, L, _ = xr.shape
    oc = O.OracleConfig.from_config(cfg)
    oc.gate_activation = m.value_gate.activation
    pos = torch.arange(L).unsqueeze(0).expand(B, -1)
    cos, sin = O.rope_cache(cfg.d_head, cfg.max_position_embeddings, cfg.rope_base, cfg.rope_scaling)
    q, k, v = O.project(W, oc, xr, pos, cos, sin)
    k_eff = sel.shape[1]
    mask = (torch.arange(k_eff).view(1, -1) < cnt.cpu().view(-1, 1)).view(B, L, k_eff)
    idx = torch.where(mask, sel.long().cpu().view(B, L, k_eff), 0)   # slots past the count are unset
    attn, _ = O.sparse_attention(q, k, v, idx, mask, cfg.n_heads // cfg.n_kv_heads, 1.0 / math.sqrt(cfg.d_head))
    g = F.linear(xr, W["output_gate.gate_proj.weight"], W["output_gate.gate_proj.bias"])
    gated = attn * O.gate_activation(g.view(B, L, cfg.n_heads, cfg.d_head), oc.gate_activation)
    out = F.linear(gated.reshape(B, L, -1), W["o_proj.weight"])
    (out * R).sum().backward()
    return out.detach(), xr.grad, {k: t.grad for k, t in W.items()}


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


DIFF = ["q_proj.weight", "k_proj.weight", "v_proj.weight", "o_proj.weight", "value_gate.gate_proj.weight",
        "value_gate.gate_proj.bias", "output_gate.gate_proj.weight", "output_gate.gate_proj.bias"]
NO_GRAD = ["indexer.q_proj.weight", "indexer.k_proj.weight", "indexer.weight_proj.weight",
           "indexer.weight_proj.bias", "indexer.bias"]


@pytest.mark.parametrize("dtype,d_model,n_heads,n_kv,HI,adaptive,gate_act,tol", [
    (torch.float32, 512, 8, 2, 4, True, "sigmoid", 1e-4),     # D = 64
    (torch.float32, 1024, 8, 2, 8, False, "tanh", 1e-4),      # D = 128, fixed k, tanh gates
    (torch.bfloat16, 1024, 8, 2, 8, True, "sigmoid", 3e-2),   # bf16 vs the fp32 gradient
])
def test_backward_matches_autograd_of_the_reference_forward(cuda_ok, dtype, d_model, n_heads, n_kv, HI, adaptive,
                                                            gate_act, tol):
    m, cfg = _layer(d_model, n_heads, n_kv, HI, dtype, adaptive, gate_act)
    B, L = 2, 320
    g = torch.Generator().manual_seed(7)
    x = torch.randn(B, L, d_model, generator=g).to(DEV, dtype).requires_grad_(True)
    R = torch.randn(B, L, d_model, generator=g)
    # the selection our forward makes (the same kernels as in the training forward)
    cap = {}
    with torch.no_grad():
        m._forward_impl(x.detach(), None, None, False, False, capture=cap)
    out = m(x)[0]
    (out.float() * R.to(DEV)).sum().backward()
    torch.cuda.synchronize()
    ref_out, ref_dx, ref_dW = _reference_grads(m, cfg, x, cap["sel"], cap["cnt"], R)
    assert _rel(out.detach(), ref_out) < (2e-5 if dtype == torch.float32 else 2e-2)
    err = _rel(x.grad, ref_dx)
    assert err < tol, ("dx", err)
    params = dict(m.named_parameters())
    for name in DIFF:
        err = _rel(params[name].grad, ref_dW[name])
        assert err < tol, (name, err)
    for name in NO_GRAD:
        assert params[name].grad is None, name


def test_backward_is_skipped_for_frozen_inputs(cuda_ok):
    """Gradients only for what requires them: a frozen layer with an input that requires grad
    gets dx and no parameter gradients."""
    m, _ = _layer(512, 8, 2, 4, torch.float32)
    for p in m.parameters():
        p.requires_grad_(False)
    x = torch.randn(1, 200, 512, device=DEV, requires_grad=True)
    m(x)[0].sum().backward()
    torch.cuda.synchronize()
    assert x.grad is not None and bool(torch.isfinite(x.grad).all())
    assert all(p.grad is None for p in m.parameters())
