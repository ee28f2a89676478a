"""Generate golden fixtures for the GSA forward path by running the reference itself.

This script imports the unmodified reference package ``gsa`` (alfredcs/Gated-Sparse-Attention)
from a checkout given by ``--reference`` (default ``/root/reference``), runs its own modules on
seeded inputs, and writes small safetensors files next to this script.  It is the only place
that executes reference code; the fixtures it writes are what the tests read.

Two shims are needed to import the reference unmodified:
  * ``gsa/__init__.py:14`` imports ``gsa/utils/checkpoint.py``, which imports ``omegaconf``
    (not installed here).  A stub module providing ``DictConfig`` and ``OmegaConf`` is created
    in a temporary directory and put first on ``sys.path``.
  * ``sys.pycache_prefix`` points at a temporary directory so that no ``.pyc`` shipped inside
    the reference checkout is ever read.

Each fixture follows the reference forward step by step
(``gsa/attention/gated_sparse_attention.py:139-232``) through the reference's own submodules,
and checks that the step-by-step output equals ``module(x, positions)`` bit for bit.

The model fixtures run the reference's GSALlamaForCausalLM (gsa/models/gsa_llama.py) the same way; the
sampling fixture runs its generate() with the model's forward replaced by seeded logits; the
adaptive fixture runs its AdaptiveTopKSelector with the entropy and learned methods.

Usage:  python tests/golden/make_golden.py [--reference PATH] [--only NAME]
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import torch
from safetensors.torch import save_file

HERE = Path(__file__).resolve().parent

# name -> (config kwargs, batch, seq_len, dtype, rows to sample or None for all rows)
FIXTURES = {
    # small shapes, every tensor stored in full
    "tiny_fp32_b2_l192": (dict(d_model=256, n_heads=4, n_kv_heads=2, d_indexer=32,
                               n_indexer_heads=4, k_base=48, k_min=16, k_max=96,
                               max_position_embeddings=1024), 2, 192, "float32", None),
    "tiny_bf16_b2_l192": (dict(d_model=256, n_heads=4, n_kv_heads=2, d_indexer=32,
                               n_indexer_heads=4, k_base=48, k_min=16, k_max=96,
                               max_position_embeddings=1024), 2, 192, "bfloat16", None),
    "tiny_fixedk_nogate_fp32_l128": (dict(d_model=256, n_heads=4, n_kv_heads=2, d_indexer=32,
                                          n_indexer_heads=2, k_base=32, k_min=16, k_max=64,
                                          use_adaptive_k=False, use_value_gate=False,
                                          use_output_gate=False,
                                          max_position_embeddings=1024), 1, 128, "float32", None),
    # the CPU-runnable 2048-token layer: d_model 512, 8/2 heads, 4 indexer heads of dim 32,
    # k_base 256 clipped to [128, 512]
    "c1_fp32_l2048": (dict(d_model=512, n_heads=8, n_kv_heads=2, d_indexer=32, n_indexer_heads=4,
                           k_base=256, k_min=128, k_max=512), 1, 2048, "float32", 24),
    # the 4096-wide layer (32/8 heads of 128, 8 indexer heads of 64) at a length the
    # reference's eager gather can hold, with k scaled down so that selection is sparse
    "w4096_bf16_l384": (dict(d_model=4096, n_heads=32, n_kv_heads=8, d_indexer=64,
                             n_indexer_heads=8, k_base=64, k_min=32, k_max=128), 1, 384,
                        "bfloat16", 24),
}

WEIGHT_SEED = 0
INPUT_SEED = 1


# name -> (config kwargs, batch, seq_len, dtype): GSALlamaForCausalLM (gsa/models/gsa_llama.py),
# every layer's output and the logits stored in full
MODEL_FIXTURES = {
    "model2_fp32_b2_l96": (dict(d_model=256, n_heads=4, n_kv_heads=2, d_indexer=32, n_indexer_heads=4,
                                k_base=24, k_min=8, k_max=48, n_layers=2, d_ffn=512, vocab_size=384,
                                max_position_embeddings=512), 2, 96, "float32"),
    "model2_bf16_b2_l96": (dict(d_model=256, n_heads=4, n_kv_heads=2, d_indexer=32, n_indexer_heads=4,
                                k_base=24, k_min=8, k_max=48, n_layers=2, d_ffn=512, vocab_size=384,
                                max_position_embeddings=512), 2, 96, "bfloat16"),
    # every row keeps all its causal keys: no selection can flip on rounding-level differences
    "model2dense_fp32_b2_l96": (dict(d_model=256, n_heads=4, n_kv_heads=2, d_indexer=32, n_indexer_heads=4,
                                     k_base=96, k_min=96, k_max=96, n_layers=2, d_ffn=512, vocab_size=384,
                                     max_position_embeddings=512), 2, 96, "float32"),
}


def _import_reference(ref_root: Path):
    tmp = Path(tempfile.mkdtemp(prefix="gsa_ref_shim_"))
    stub = tmp / "omegaconf"
    stub.mkdir()
    (stub / "__init__.py").write_text(
        "class DictConfig(dict):\n    pass\n\n"
        "class OmegaConf:\n    @staticmethod\n    def to_container(cfg, resolve=True):\n"
        "        return dict(cfg)\n")
    sys.pycache_prefix = str(tmp / "pycache")
    sys.path.insert(0, str(tmp))
    sys.path.insert(0, str(ref_root))
    import gsa  # noqa: F401  (the reference package)
    from gsa import GSAConfig, GatedSparseAttention
    from gsa.attention.rope import apply_rotary_pos_emb
    from gsa.models.gsa_llama import GSALlamaForCausalLM
    return GSAConfig, GatedSparseAttention, apply_rotary_pos_emb, GSALlamaForCausalLM


def _sample_rows(L: int, n: int | None):
    if n is None:
        return torch.arange(L)
    head = [0, 1, 2, 3, 7, 15, 31, 63]
    rest = torch.linspace(64, L - 1, n - len(head)).round().long().tolist()
    rows = sorted(set(h for h in head if h < L) | set(rest))
    return torch.tensor(rows, dtype=torch.long)


def _checksums(module) -> dict:
    out = {}
    for name, p in module.state_dict().items():
        t = p.detach().double()
        out[name] = [float(t.sum()), float((t * t).sum()), [float(v) for v in t.flatten()[:4]]]
    return out


@torch.no_grad()
def make_fixture(name, spec, refs):
    GSAConfig, GatedSparseAttention, apply_rotary_pos_emb, _ = refs
    cfg_kwargs, B, L, dtype_name, n_rows = spec
    dtype = getattr(torch, dtype_name)
    cfg = GSAConfig(**cfg_kwargs)

    torch.manual_seed(WEIGHT_SEED)
    m = GatedSparseAttention(cfg).eval()
    m = m.to(dtype)
    gen = torch.Generator().manual_seed(INPUT_SEED)
    x = torch.randn(B, L, cfg.d_model, generator=gen).to(dtype)
    positions = torch.arange(L).unsqueeze(0).expand(B, -1)

    # reference forward, step by step (gated_sparse_attention.py:167-230)
    q = m.q_proj(x).view(B, L, m.n_heads, m.d_head)
    k = m.k_proj(x).view(B, L, m.n_kv_heads, m.d_head)
    v = m.v_proj(x).view(B, L, m.n_kv_heads, m.d_head)
    if m.value_gate is not None:
        v = m.value_gate(v, x)
    cos, sin = m.rotary_emb(positions)
    q, k = apply_rotary_pos_emb(q, k, cos, sin)
    scores = m.indexer(x, positions, kv_hidden_states=None)
    indices, mask, k_values = m.topk_selector(scores, L, scores.shape[-1], return_k_values=True)
    attn, _ = m._sparse_attention(q, k, v, indices, mask)
    gated = m.output_gate(attn, x) if m.output_gate is not None else attn
    out = m.o_proj(gated.reshape(B, L, -1))

    full, _, _ = m(x, positions=positions)
    assert torch.equal(full, out), f"{name}: step-by-step forward differs from module forward"

    # the per-row variance exactly as adaptive_topk.py:84-93 computes it
    valid = scores != float("-inf")
    var = scores.masked_fill(~valid, 0).var(dim=-1)

    rows = _sample_rows(L, n_rows)
    t = {
        "rows": rows.to(torch.int32),
        "k_values": k_values.to(torch.int32),
        "var": var,
        "q": q[:, rows].contiguous(),
        "k": k.contiguous() if n_rows is None else k[:, rows].contiguous(),
        "v": v.contiguous() if n_rows is None else v[:, rows].contiguous(),
        "scores": scores[:, rows].contiguous(),
        "indices": indices[:, rows].to(torch.int32).contiguous(),
        "mask": mask[:, rows].to(torch.uint8).contiguous(),
        "attn": attn[:, rows].contiguous(),
        "out": out[:, rows].contiguous(),
    }
    if n_rows is None:
        t["x"] = x.contiguous()
    meta = {
        "config": json.dumps(cfg_kwargs),
        "batch": str(B),
        "seq_len": str(L),
        "dtype": dtype_name,
        "weight_seed": str(WEIGHT_SEED),
        "input_seed": str(INPUT_SEED),
        "param_checksums": json.dumps(_checksums(m)),
        "x_checksum": json.dumps([float(x.double().sum()), float((x.double() ** 2).sum())]),
        "var_mean": repr(float(var.mean())),
        "torch": torch.__version__,
    }
    path = HERE / f"{name}.safetensors"
    save_file(t, str(path), metadata=meta)
    print(f"{name}: {path.stat().st_size / 1024:.0f} KiB, k_values mean "
          f"{k_values.float().mean():.1f}, rows {len(rows)}")


@torch.no_grad()
def make_model_fixture(name, spec, refs):
    """GSALlamaForCausalLM forward (gsa_llama.py:164-242, 278-330) on seeded token ids, stepping
    through the reference's own modules; the step-by-step logits must equal model(input_ids)."""
    GSAConfig, _, _, GSALlamaForCausalLM = refs
    cfg_kwargs, B, L, dtype_name = spec
    dtype = getattr(torch, dtype_name)
    cfg = GSAConfig(**cfg_kwargs)
    torch.manual_seed(WEIGHT_SEED)
    model = GSALlamaForCausalLM(cfg).eval().to(dtype)
    # distinct token ids: a repeated token has the same indexer key (k^I carries no position), so
    # its scores tie exactly and torch.topk would break the tie at a k_t boundary arbitrarily
    gen = torch.Generator().manual_seed(INPUT_SEED)
    ids = torch.randperm(cfg.vocab_size, generator=gen)[:B * L].view(B, L)
    positions = torch.arange(L).unsqueeze(0).expand(B, -1)
    h = model.model.embed_tokens(ids)
    t = {"input_ids": ids.to(torch.int32), "embed": h.contiguous()}
    for i, layer in enumerate(model.model.layers):
        normed = layer.input_layernorm(h)
        attn, _, _ = layer.self_attn(normed, positions=positions)
        h1 = h + attn
        normed2 = layer.post_attention_layernorm(h1)
        h = h1 + layer.mlp(normed2)
        t[f"layer{i}_normed"] = normed.contiguous()
        t[f"layer{i}_attn"] = attn.contiguous()
        t[f"layer{i}_out"] = h.contiguous()
    h = model.model.norm(h)
    logits = model.lm_head(h)
    full = model(ids).logits
    assert torch.equal(full, logits), f"{name}: step-by-step logits differ from model(input_ids)"
    t["logits"] = logits.contiguous()
    meta = {
        "config": json.dumps(cfg_kwargs),
        "batch": str(B),
        "seq_len": str(L),
        "dtype": dtype_name,
        "weight_seed": str(WEIGHT_SEED),
        "input_seed": str(INPUT_SEED),
        "param_checksums": json.dumps(_checksums(model)),
        "torch": torch.__version__,
    }
    path = HERE / f"{name}.safetensors"
    save_file(t, str(path), metadata=meta)
    print(f"{name}: {path.stat().st_size / 1024:.0f} KiB")


# name -> (batch, vocab, prompt length, steps, [(temperature, top_k, top_p, do_sample, seed), ...])
SAMPLING_FIXTURES = {
    "sampling_b3_v96": (3, 96, 5, 12, [(1.0, 50, 0.9, True, 11), (0.7, 8, 0.8, True, 12), (1.3, 0, 0.5, True, 13),
                                       (1.0, 20, 1.0, True, 14), (1.0, 50, 0.9, False, 15)]),
}


def make_sampling_fixture(name, spec, refs):
    """The reference's GSALlamaForCausalLM.generate (gsa_llama.py:344-430) with its forward replaced
    by a stub that returns seeded logits, one [B, 1, V] block per step: what is recorded is the
    sampling alone -- temperature, top-k, top-p filtering and torch.multinomial / argmax -- for
    several settings, each under torch.manual_seed(seed) before the call.  The logits are quantised
    to quarters, so equal values (ties at the top-k and top-p cuts) occur."""
    GSAConfig, _, _, GSALlamaForCausalLM = refs
    B, V, P, steps, settings = spec
    cfg = GSAConfig(d_model=64, n_heads=2, n_kv_heads=1, d_indexer=16, n_indexer_heads=2, k_base=8, k_min=4,
                    k_max=16, n_layers=1, d_ffn=128, vocab_size=V, max_position_embeddings=64)
    torch.manual_seed(WEIGHT_SEED)
    model = GSALlamaForCausalLM(cfg).eval()
    gen = torch.Generator().manual_seed(INPUT_SEED)
    logits = (torch.randn(steps, B, 1, V, generator=gen) * 8).round() / 4
    prompt = torch.randint(0, V, (B, P), generator=gen)
    calls = []

    class _Out:
        def __init__(self, lg):
            self.logits = lg
            self.past_key_values = ("cache",)

    def stub(input_ids=None, past_key_values=None, use_cache=False, **kw):
        i = len(calls)
        calls.append(int(input_ids.shape[1]))
        return _Out(logits[i].clone())

    model.forward = stub
    t = {"logits": logits.contiguous(), "prompt": prompt.to(torch.int32)}
    for j, (temp, top_k, top_p, do_sample, seed) in enumerate(settings):
        calls.clear()
        torch.manual_seed(seed)
        out = model.generate(prompt, max_new_tokens=steps, temperature=temp, top_p=top_p, top_k=top_k,
                             do_sample=do_sample)
        assert calls == [P] + [1] * (steps - 1), calls
        t[f"tokens{j}"] = out.to(torch.int32).contiguous()
    meta = {"settings": json.dumps(settings), "batch": str(B), "vocab": str(V), "steps": str(steps),
            "torch": torch.__version__}
    path = HERE / f"{name}.safetensors"
    save_file(t, str(path), metadata=meta)
    print(f"{name}: {path.stat().st_size / 1024:.0f} KiB")


# name -> (batch, seq_len, k_base, k_min, k_max, temperatures): the reference's AdaptiveTopKSelector
# with adaptive_method "entropy" and "learned" (adaptive_topk.py:84-133), which the attention layer
# never selects but the selector module offers
ADAPTIVE_FIXTURES = {
    "adaptive_methods_b2_l96": (2, 96, 48, 16, 80, [1.0, 0.6]),
}


def make_adaptive_fixture(name, spec, ref_root: Path):
    """k_t of the reference selector's entropy and learned methods on seeded indexer-like scores
    (values in [0, 3], causal -inf mask), fp32 and bf16.  The learned method's predictor is the
    selector's own seeded initialisation (torch.manual_seed(WEIGHT_SEED) before construction); its
    weights are stored too."""
    from gsa.attention.adaptive_topk import AdaptiveTopKSelector
    B, L, k_base, k_min, k_max, temps = spec
    gen = torch.Generator().manual_seed(INPUT_SEED)
    base = torch.rand(B, L, L, generator=gen) * 3
    causal = torch.triu(torch.ones(L, L, dtype=torch.bool), diagonal=1)
    base = base.masked_fill(causal, float("-inf"))
    t = {}
    for dname in ("float32", "bfloat16"):
        dt = getattr(torch, dname)
        scores = base.to(dt)
        t[f"scores_{dname}"] = scores.clone().contiguous()
        for method in ("entropy", "learned"):
            for j, temp in enumerate(temps):
                torch.manual_seed(WEIGHT_SEED)
                sel = AdaptiveTopKSelector(k_base=k_base, k_min=k_min, k_max=k_max, use_adaptive=True,
                                           temperature=temp, adaptive_method=method).to(dt)
                with torch.no_grad():
                    _, _, kv = sel(scores, L, L, return_k_values=True)
                t[f"k_{method}_{dname}_t{j}"] = kv.to(torch.int32).contiguous()
                if method == "learned" and j == 0:
                    for pn, pv in sel.k_predictor.state_dict().items():
                        t[f"pred_{dname}.{pn}"] = pv.clone().contiguous()
    meta = {"batch": str(B), "seq_len": str(L), "k_base": str(k_base), "k_min": str(k_min),
            "k_max": str(k_max), "temperatures": json.dumps(temps), "torch": torch.__version__}
    path = HERE / f"{name}.safetensors"
    save_file(t, str(path), metadata=meta)
    print(f"{name}: {path.stat().st_size / 1024:.0f} KiB")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("GSA_REFERENCE", "/root/reference"))
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 1)
    refs = _import_reference(Path(args.reference))
    for name, spec in FIXTURES.items():
        if args.only and name != args.only:
            continue
        make_fixture(name, spec, refs)
    for name, spec in MODEL_FIXTURES.items():
        if args.only and name != args.only:
            continue
        make_model_fixture(name, spec, refs)
    for name, spec in SAMPLING_FIXTURES.items():
        if args.only and name != args.only:
            continue
        make_sampling_fixture(name, spec, refs)
    for name, spec in ADAPTIVE_FIXTURES.items():
        if args.only and name != args.only:
            continue
        make_adaptive_fixture(name, spec, Path(args.reference))


if __name__ == "__main__":
    main()
