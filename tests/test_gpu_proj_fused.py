"""The fused projection GEMM (gsa_proj_fused: tcgen05 GEMM with RoPE, G2, the G1 gate, q^I / k^I and
w = sigmoid(.) in its epilogue) against the unfused pair it replaces -- the cuBLAS GEMM
proj = x . Wcat^T + b and gsa_proj_epilogue -- on the same inputs (gated_sparse_attention.py:175-186,
value_gate.py:95-113, output_gate.py:101-117, gated_indexer.py:114-121, rope.py:151-185).

Both round the projection to bf16 before the epilogue's ops, which are the same ops in the same
order; they differ only in the GEMM's fp32 summation order, which moves a bf16 projection value by
one unit in the last place now and then.  So: every output tensor within 4e-3 (relative, Frobenius)
of the unfused one and at least 97% of its elements bit-identical; w and shift within 1e-3.
Shapes: the 4096-wide layer (d_head 128) at 1000 tokens (a ragged last row block), two sequences
written into a KV cache with room (batch strides), and a d_head-64 layer."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _layer(d_model, H, Hk, HI, dI, seed=0):
    from gsa_b200 import GSAConfig, GatedSparseAttention

    cfg = GSAConfig(d_model=d_model, n_heads=H, n_kv_heads=Hk, d_indexer=dI, n_indexer_heads=HI, k_base=64,
                    k_min=32, k_max=128, max_position_embeddings=4096)
    torch.manual_seed(seed)
    return GatedSparseAttention(cfg).eval().to(torch.bfloat16).to(DEV)


def _compare(m, B, L, past=0, cap=None):
    from gsa_b200 import ops
    from gsa_b200.attention import KVCacheStore

    H, Hk, D = m.n_heads, m.n_kv_heads, m.d_head
    HI, dI = m.config.n_indexer_heads, m.config.d_indexer
    x = torch.randn(B * L, m.d_model, generator=torch.Generator().manual_seed(5)).to(DEV, torch.bfloat16)
    pos = (torch.arange(L, device=DEV) + past).unsqueeze(0).expand(B, -1)
    dims = m._step_constants()[0]
    W, bvec, layout = m.fused_projection()
    proj = torch.addmm(bvec, x, W.t())
    ref_store = KVCacheStore(B, cap, Hk, D, dI, torch.bfloat16, DEV) if cap else None
    store = KVCacheStore(B, cap, Hk, D, dI, torch.bfloat16, DEV) if cap else None
    if cap:
        store.kv.zero_()
        store.ki.zero_()
    q0, kv0, g10, w0, s0 = ops.proj_epilogue(
        dims, layout, proj, pos, m.rotary_emb.cos_cached, m.rotary_emb.sin_cached, True, return_kv=True,
        kv_out=ref_store.kv[:, past:past + L] if cap else None, ki_out=ref_store.ki[:, past:past + L] if cap else None)
    qi0 = proj.view(B, L, -1)[..., layout.qi:layout.qi + HI * dI]
    ki0 = ref_store.ki[:, past:past + L] if cap else proj.view(B, L, -1)[..., layout.ki:layout.ki + dI]
    Wp, bp = m.fused_projection_tiles()
    out = ops.proj_fused(dims, Wp, bp, x, B, L, pos, m.rotary_emb.cos_cached, m.rotary_emb.sin_cached,
                         kv_out=store.kv[:, past:past + L] if cap else None,
                         ki_out=store.ki[:, past:past + L] if cap else None)
    torch.cuda.synchronize()
    ops.check_device_error()
    assert out is not None, "the fused projection GEMM declined these shapes"
    q, kv, g1, w, s, qi, ki = out
    pairs = [("q", q, q0), ("k", kv[:, :, 0], kv0.view(B, L, 2, Hk, D)[:, :, 0]),
             ("v", kv[:, :, 1], kv0.view(B, L, 2, Hk, D)[:, :, 1]), ("g1", g1, g10), ("qI", qi, qi0), ("kI", ki, ki0)]
    for name, a, b in pairs:
        e = rel(a, b)
        same = float((a == b).double().mean())
        print(f"{name}: rel {e:.2e}, identical {same:.4f}")
        assert e < 4e-3, (name, e)
        assert same >= 0.97, (name, same)
    assert rel(w, w0) < 1e-3 and rel(s, s0) < 1e-3
    if cap:
        # nothing outside the new tokens' slots was written
        assert bool((store.kv[:, :past] == 0).all()) and bool((store.kv[:, past + L:] == 0).all())


def test_fused_projection_4096_wide_ragged_rows(cuda_ok):
    _compare(_layer(4096, 32, 8, 8, 64), 1, 1000)


def test_fused_projection_into_a_kv_cache(cuda_ok):
    _compare(_layer(4096, 32, 8, 8, 64), 2, 300, past=17, cap=400)


def test_fused_projection_head_dim_64(cuda_ok):
    _compare(_layer(1024, 16, 4, 4, 64), 2, 256)


def test_layer_fused_and_unfused_agree(cuda_ok):
    """The whole bf16 layer with the fused GEMM equals the layer with cuBLAS + the epilogue kernel,
    up to the projection's summation order (which can move a bf16 selection tie)."""
    from gsa_b200 import ops

    m = _layer(4096, 32, 8, 8, 64)
    x = torch.randn(1, 2048, 4096, generator=torch.Generator().manual_seed(9)).to(DEV, torch.bfloat16)
    with torch.no_grad():
        fused, _, _ = m(x)
        m.fused_gemm = False
        plain, _, _ = m(x)
        m.fused_gemm = True
    torch.cuda.synchronize()
    ops.check_device_error()
    e = rel(fused, plain)
    print(f"layer output fused vs unfused: rel {e:.2e}")
    assert e < 1e-2
    # the gates' scores are still there when read (computed from the input on demand)
    g = m.output_gate.last_gate_scores
    assert g is not None and g.shape == (1, 2048, 32, 128) and bool(((g >= 0) & (g <= 1)).all())
