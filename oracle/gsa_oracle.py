"""CPU oracle for the GSA attention forward path -- TEST INFRASTRUCTURE ONLY.

This module restates, in PyTorch CPU ops, the algorithm of the reference
alfredcs/Gated-Sparse-Attention forward path (``GatedSparseAttention.forward``,
``gsa/attention/gated_sparse_attention.py:139-232``) so that the CUDA path can be checked
against it.  It is pinned against golden fixtures produced by running the reference itself
(``tests/golden/make_golden.py``); the pinning tests live in ``tests/test_oracle_golden.py``.

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
this module.  The product path never calls it.

Every function follows the same torch ops, in the same order and dtype, as the reference lines
it cites, with one structural change the reference's own eager code cannot do without: the
indexer, the top-k and the sparse attention run over chunks of query rows with an explicit
offset-causal mask, so that no ``[B, L, L]`` tensor is needed for long sequences.  Chunking
is exact: each query row's scores, variance and selection depend only on that row, and the
adaptive-k mean is taken over all rows after every chunk's variance is known.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

NEG_INF = float("-inf")


# --------------------------------------------------------------------------------------------
# RoPE  (gsa/attention/rope.py)
# --------------------------------------------------------------------------------------------
def rope_inv_freq(dim: int, base: float, scaling: dict | None) -> torch.Tensor:
    """Inverse frequencies; rope.py:45-101 (standard, ntk, yarn; dynamic_ntk == standard)."""
    scaling = scaling or {}
    kind = scaling.get("type", None)
    ar = torch.arange(0, dim, 2).float()
    if kind == "ntk":  # rope.py:66-71
        factor = scaling.get("factor", 1.0)
        b = base * factor ** (dim / (dim - 2))
        return 1.0 / (b ** (ar / dim))
    if kind == "yarn":  # rope.py:73-101
        factor = scaling.get("factor", 1.0)
        orig = scaling.get("original_max_position_embeddings", 4096)
        beta_fast = scaling.get("beta_fast", 32)
        beta_slow = scaling.get("beta_slow", 1)
        pos_freqs = base ** (ar / dim)
        extra = 1.0 / pos_freqs
        inter = 1.0 / (factor * pos_freqs)
        low = max(int(math.floor(dim * math.log(orig / (beta_fast * 2 * math.pi))
                                 / (2 * math.log(base)))), 0)
        high = min(int(math.ceil(dim * math.log(orig / (beta_slow * 2 * math.pi))
                                 / (2 * math.log(base)))), dim // 2 - 1)
        inv = inter.clone()
        inv[:low] = extra[:low]
        if high > low:
            smooth = (torch.arange(low, high + 1).float() - low) / (high - low)
            inv[low:high + 1] = (1 - smooth) * extra[low:high + 1] + smooth * inter[low:high + 1]
        return inv
    return 1.0 / (base ** (ar / dim))  # rope.py:59-64


def rope_cache(dim: int, max_pos: int, base: float, scaling: dict | None):
    """cos/sin tables [max_pos, dim] in fp32; rope.py:103-115."""
    inv = rope_inv_freq(dim, base, scaling)
    t = torch.arange(max_pos, dtype=torch.float32)
    freqs = torch.outer(t, inv)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """rotate-half RoPE; rope.py:151-185.  x [B,L,H,D], cos/sin [B,L,D]."""
    cos = cos.unsqueeze(2)
    sin = sin.unsqueeze(2)
    half = x.shape[-1] // 2
    rotated = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rotated * sin


# --------------------------------------------------------------------------------------------
# Gates  (gsa/attention/value_gate.py, output_gate.py)
# --------------------------------------------------------------------------------------------
def gate_activation(logits: torch.Tensor, activation: str) -> torch.Tensor:
    """value_gate.py:98-106 / output_gate.py:111-119."""
    if activation == "sigmoid":
        return torch.sigmoid(logits)
    if activation == "tanh":
        return (torch.tanh(logits) + 1) / 2
    if activation == "silu":
        return F.silu(logits)
    raise ValueError(f"Unknown activation: {activation}")


# --------------------------------------------------------------------------------------------
# Indexer  (gsa/attention/gated_indexer.py:106-155)
# --------------------------------------------------------------------------------------------
def indexer_scores(W: dict, x_q: torch.Tensor, x_kv: torch.Tensor, n_heads: int, d_idx: int,
                   activation: str = "sigmoid", q_offset: int | None = 0) -> torch.Tensor:
    """Gated indexer scores for query rows ``x_q`` against keys ``x_kv``.

    Follows gated_indexer.py:114-145 op for op.  The causal mask of gated_indexer.py:148-153
    (``triu(diagonal=1)`` when ``seq_q == seq_kv``) is restated with an offset: query row i of
    the chunk has absolute position ``q_offset + i`` and key s is masked when
    ``s > q_offset + i``.  ``q_offset=None`` disables the mask (the reference's behaviour when
    ``seq_q != seq_kv``).
    """
    B, Lq, _ = x_q.shape
    q_idx = F.linear(x_q, W["indexer.q_proj.weight"]).view(B, Lq, n_heads, d_idx)
    k_idx = F.linear(x_kv, W["indexer.k_proj.weight"])
    weights = torch.sigmoid(F.linear(x_q, W["indexer.weight_proj.weight"],
                                     W["indexer.weight_proj.bias"]))
    return indexer_scores_from_proj(q_idx, k_idx, weights, W["indexer.bias"], activation, q_offset)


def indexer_scores_from_proj(q_idx, k_idx, weights, bias_param, activation="sigmoid",
                             q_offset: int | None = 0) -> torch.Tensor:
    """gated_indexer.py:123-153 from the projected q^I [B,Lq,H_I,d_I], k^I [B,Lkv,d_I] and the
    head weights sigmoid(weight_proj(h)) [B,Lq,H_I]; offset-causal as in indexer_scores."""
    B, Lq, _, d_idx = q_idx.shape
    Lkv = k_idx.shape[1]
    raw = torch.einsum("bqhd,bkd->bhqk", q_idx, k_idx) * (1.0 / math.sqrt(d_idx))
    bias = bias_param.view(1, -1, 1, 1)
    if activation == "sigmoid":
        gated = torch.sigmoid(raw + bias)
    elif activation == "relu":
        gated = F.relu(raw + bias)
    else:
        raise ValueError(f"Unknown activation: {activation}")
    scores = (gated * weights.permute(0, 2, 1).unsqueeze(-1)).sum(dim=1)
    if q_offset is not None:
        t = torch.arange(Lq).view(-1, 1) + q_offset
        s = torch.arange(Lkv).view(1, -1)
        scores = scores.masked_fill((s > t).unsqueeze(0), NEG_INF)
    return scores


# --------------------------------------------------------------------------------------------
# Adaptive top-k  (gsa/attention/adaptive_topk.py)
# --------------------------------------------------------------------------------------------
def row_variance(scores: torch.Tensor):
    """Per-row unbiased variance with -inf entries counted as 0; adaptive_topk.py:84-93.

    Returns (var [B,Lq] in the scores' dtype, valid_counts [B,Lq] float32).
    """
    valid = scores != NEG_INF
    var = scores.masked_fill(~valid, 0).var(dim=-1)
    return var, valid.sum(dim=-1).float()


def adaptive_k(var: torch.Tensor, valid_counts: torch.Tensor, var_mean: torch.Tensor,
               k_base: int, k_min: int, k_max: int, temperature: float) -> torch.Tensor:
    """k_t from the variance; adaptive_topk.py:96-102 and :132-136 (``variance`` method).

    ``var_mean`` is ``score_var.mean()`` over every (batch, query) row of the layer call,
    computed by the caller once all chunks are known (adaptive_topk.py:96).
    """
    var_normalized = var / (var_mean + 1e-8)
    k_scale = 1.0 / (1.0 + var_normalized * temperature)
    k_adaptive = k_base * (0.5 + k_scale)
    k_values = torch.clamp(k_adaptive, k_min, k_max)
    k_values = torch.minimum(k_values, valid_counts)
    return k_values.long()


def adaptive_k_prefloor(var, valid_counts, var_mean, k_base, k_min, k_max, temperature):
    """The float value :func:`adaptive_k` truncates, for boundary reporting in tests."""
    var_normalized = var / (var_mean + 1e-8)
    k_scale = 1.0 / (1.0 + var_normalized * temperature)
    k_values = torch.clamp(k_base * (0.5 + k_scale), k_min, k_max)
    return torch.minimum(k_values, valid_counts)


def adaptive_k_method(scores: torch.Tensor, method: str, k_base: int, k_min: int, k_max: int,
                      temperature: float, predictor=None) -> torch.Tensor:
    """k_t of the ``entropy`` and ``learned`` methods; adaptive_topk.py:84-90 (masks and counts),
    :104-117 (entropy: softmax entropy of the valid scores over log(count + 1)), :119-127 (learned:
    [mean, std, max] of the masked scores through the selector's predictor) and :129-133 (clamp).
    The selector's forward never mixes rows, so rows may come in any grouping."""
    valid = scores != NEG_INF
    masked = scores.masked_fill(~valid, 0)
    valid_counts = valid.sum(dim=-1).float()
    if method == "entropy":
        probs = torch.softmax(masked.masked_fill(~valid, NEG_INF), dim=-1).masked_fill(~valid, 0)
        entropy = -(probs * torch.log(probs + 1e-10)).sum(dim=-1)
        normalized = entropy / (torch.log(valid_counts + 1) + 1e-8)
        k_adaptive = k_base * (0.5 + normalized * temperature)
    elif method == "learned":
        stats = torch.cat([masked.mean(dim=-1, keepdim=True), masked.std(dim=-1, keepdim=True),
                           masked.max(dim=-1, keepdim=True).values], dim=-1)
        k_adaptive = k_min + predictor(stats).squeeze(-1) * (k_max - k_min)
    else:
        raise ValueError(f"Unknown adaptive method: {method}")
    return torch.minimum(torch.clamp(k_adaptive, k_min, k_max), valid_counts).long()


def adaptive_method_predictor(state: dict, dtype=torch.float32) -> torch.nn.Module:
    """The learned method's predictor (adaptive_topk.py:60-66: Linear(3, 32), ReLU, Linear(32, 1),
    Sigmoid) holding the given weights."""
    net = torch.nn.Sequential(torch.nn.Linear(3, 32), torch.nn.ReLU(), torch.nn.Linear(32, 1), torch.nn.Sigmoid())
    net.load_state_dict(state)
    return net.to(dtype)


def topk_select(scores: torch.Tensor, k_eff: int, k_values: torch.Tensor):
    """adaptive_topk.py:174-189: sorted top-k_eff, mask p < k_t and score != -inf."""
    B, Lq, _ = scores.shape
    scores_for_topk = scores.masked_fill(scores == NEG_INF, -1e9)
    _, indices = torch.topk(scores_for_topk, k_eff, dim=-1)
    pos = torch.arange(k_eff).view(1, 1, -1).expand(B, Lq, -1)
    mask = pos < k_values.unsqueeze(-1)
    mask = mask & (torch.gather(scores, -1, indices) != NEG_INF)
    return indices, mask


def topk_sets_stable(scores: torch.Tensor, k_values: torch.Tensor):
    """The index set each row keeps, with ties broken lower index first.

    Same selection rule as :func:`topk_select` (the top ``k_t`` finite scores), but with a
    defined tie order: scores descending, then index ascending.  Returns a list over rows of
    sorted int64 numpy arrays; ``scores`` is [R, Lkv] and ``k_values`` [R].
    """
    s = scores.detach().float().numpy()
    kv = k_values.detach().numpy().astype(np.int64)
    out = []
    for r in range(s.shape[0]):
        row = s[r]
        finite = np.flatnonzero(row != -np.inf)
        order = finite[np.lexsort((finite, -row[finite]))]
        out.append(np.sort(order[: max(0, min(int(kv[r]), len(order)))]))
    return out


def boundary_tie_rows(scores: torch.Tensor, k_values: torch.Tensor) -> np.ndarray:
    """Rows whose k_t-th and (k_t+1)-th largest finite scores are equal (a tie at the cut)."""
    s = scores.detach().float().numpy()
    kv = k_values.detach().numpy().astype(np.int64)
    bad = []
    for r in range(s.shape[0]):
        row = s[r][s[r] != -np.inf]
        k = int(kv[r])
        if 0 < k < len(row):
            srt = np.sort(row)[::-1]
            if srt[k - 1] == srt[k]:
                bad.append(r)
    return np.array(bad, dtype=np.int64)


# --------------------------------------------------------------------------------------------
# Sparse attention  (gsa/attention/gated_sparse_attention.py:123-137, 234-323)
# --------------------------------------------------------------------------------------------
def sparse_attention(q, k, v, indices, mask, n_rep: int, scale: float):
    """GQA sparse SDPA over one index set per (b, t) shared by all heads.

    q [B,Lq,H,D]; k, v [B,Lkv,Hk,D]; indices, mask [B,Lq,ksel].  Restates
    ``_repeat_kv`` (:123-137), ``_gather_along_seq`` (:292-323) and ``_sparse_attention``
    (:256-290) with dropout off (eval).  Returns (output [B,Lq,H,D], weights [B,Lq,H,ksel]).
    """
    B, Lq, H, D = q.shape
    Lkv = k.shape[1]
    if n_rep > 1:
        k = k.unsqueeze(3).expand(B, Lkv, k.shape[2], n_rep, D).reshape(B, Lkv, H, D)
        v = v.unsqueeze(3).expand(B, Lkv, v.shape[2], n_rep, D).reshape(B, Lkv, H, D)
    ksel = indices.shape[-1]
    idx = indices.unsqueeze(-1).unsqueeze(-1).expand(B, Lq, ksel, H, D)
    kg = torch.gather(k.unsqueeze(1).expand(B, Lq, Lkv, H, D), 2, idx).permute(0, 1, 3, 2, 4)
    vg = torch.gather(v.unsqueeze(1).expand(B, Lq, Lkv, H, D), 2, idx).permute(0, 1, 3, 2, 4)
    scores = torch.einsum("bqhd,bqhkd->bqhk", q, kg) * scale
    m = mask.unsqueeze(2)
    scores = scores.masked_fill(~m, NEG_INF)
    w = F.softmax(scores, dim=-1)
    w = w.masked_fill(~m, 0.0)
    out = torch.einsum("bqhk,bqhkd->bqhd", w, vg)
    return out, w


# --------------------------------------------------------------------------------------------
# Full layer
# --------------------------------------------------------------------------------------------
@dataclass
class OracleConfig:
    d_model: int
    n_heads: int
    n_kv_heads: int
    d_head: int
    d_indexer: int
    n_indexer_heads: int
    k_base: int
    k_min: int
    k_max: int
    use_adaptive_k: bool = True
    adaptive_k_temperature: float = 1.0
    use_value_gate: bool = True
    use_output_gate: bool = True
    gate_activation: str = "sigmoid"
    indexer_activation: str = "sigmoid"
    rope_base: float = 10000.0
    rope_scaling: dict | None = None
    max_position_embeddings: int = 131072
    gate_bias_init: float = 0.5

    @classmethod
    def from_config(cls, cfg) -> "OracleConfig":
        """The layer the reference builds from a GSAConfig.  GatedSparseAttention does not pass
        config.gate_activation to its ValueGate / OutputGate (gated_sparse_attention.py:81-99),
        so both gates use their default sigmoid (value_gate.py:43, output_gate.py:46) whatever
        the config says; set gate_activation on the result to model gates built otherwise."""
        d = {f: getattr(cfg, f) for f in cls.__dataclass_fields__}
        d["gate_activation"] = "sigmoid"
        return cls(**d)


def init_layer_weights(cfg: OracleConfig, seed: int, n_layers: int = 32, dtype=torch.float32) -> dict:
    """The parameters ``torch.manual_seed(seed); GatedSparseAttention(config)`` creates, by name.

    Restates the construction order of gated_sparse_attention.py:57-121 with torch's own
    ``nn.Linear`` (whose default init draws from the global generator): q/k/v/o projections
    (:57-61), the indexer's three projections and bias, initialised inside its constructor
    (gated_indexer.py:65-86), the value gate (value_gate.py:65-75) and the output gate
    (output_gate.py:68-84, per head; both biases at gate_bias_init, :81-99), then the layer's xavier gains for q/k/v (1/sqrt 2) and o
    (1/sqrt(2 n_layers), :116-121).  ``n_layers`` is the config field (32 by default)."""
    torch.manual_seed(seed)
    H, Hk, D, d = cfg.n_heads, cfg.n_kv_heads, cfg.d_head, cfg.d_model
    HI, dI = cfg.n_indexer_heads, cfg.d_indexer
    lin = torch.nn.Linear
    q, k, v, o = lin(d, H * D, bias=False), lin(d, Hk * D, bias=False), lin(d, Hk * D, bias=False), \
        lin(H * D, d, bias=False)
    iq, ik, iw = lin(d, HI * dI, bias=False), lin(d, dI, bias=False), lin(d, HI, bias=True)
    ibias = torch.zeros(HI)
    torch.nn.init.xavier_uniform_(iq.weight, gain=1.0)
    torch.nn.init.xavier_uniform_(ik.weight, gain=1.0)
    torch.nn.init.xavier_uniform_(iw.weight, gain=0.1)
    torch.nn.init.zeros_(iw.bias)
    W = {"indexer.q_proj.weight": iq.weight, "indexer.k_proj.weight": ik.weight,
         "indexer.weight_proj.weight": iw.weight, "indexer.weight_proj.bias": iw.bias, "indexer.bias": ibias}
    for name, use, width in (("value_gate", cfg.use_value_gate, Hk * D), ("output_gate", cfg.use_output_gate, H * D)):
        if use:
            g = lin(d, width, bias=True)
            torch.nn.init.xavier_uniform_(g.weight, gain=0.1)
            torch.nn.init.constant_(g.bias, cfg.gate_bias_init)
            W[f"{name}.gate_proj.weight"], W[f"{name}.gate_proj.bias"] = g.weight, g.bias
    for name, m in (("q_proj", q), ("k_proj", k), ("v_proj", v)):
        torch.nn.init.xavier_uniform_(m.weight, gain=1.0 / math.sqrt(2))
        W[f"{name}.weight"] = m.weight
    torch.nn.init.xavier_uniform_(o.weight, gain=1.0 / math.sqrt(2 * n_layers))
    W["o_proj.weight"] = o.weight
    return {kk: vv.detach().to(dtype) for kk, vv in W.items()}


def project(W: dict, cfg: OracleConfig, x: torch.Tensor, positions: torch.Tensor,
            cos_cached: torch.Tensor, sin_cached: torch.Tensor):
    """q/k/v projections, G2 and RoPE; gated_sparse_attention.py:175-186, value_gate.py:95-113.

    ``cos_cached``/``sin_cached`` are the module's buffers (fp32, or bf16 after ``.to``)."""
    B, L, _ = x.shape
    H, Hk, D = cfg.n_heads, cfg.n_kv_heads, cfg.d_head
    q = F.linear(x, W["q_proj.weight"]).view(B, L, H, D)
    k = F.linear(x, W["k_proj.weight"]).view(B, L, Hk, D)
    v = F.linear(x, W["v_proj.weight"]).view(B, L, Hk, D)
    if cfg.use_value_gate:
        g = F.linear(x, W["value_gate.gate_proj.weight"], W["value_gate.gate_proj.bias"])
        v = v * gate_activation(g.view(B, L, Hk, D), cfg.gate_activation)
    cos = cos_cached[positions]
    sin = sin_cached[positions]
    return apply_rope(q, cos, sin), apply_rope(k, cos, sin), v


def k_effective(cfg: OracleConfig, seq_kv: int) -> int:
    """adaptive_topk.py:161-172."""
    return min(cfg.k_max, seq_kv) if cfg.use_adaptive_k else min(cfg.k_base, seq_kv)


def gsa_forward(W: dict, cfg: OracleConfig, x: torch.Tensor, positions: torch.Tensor | None = None,
                cos_cached: torch.Tensor | None = None, sin_cached: torch.Tensor | None = None,
                chunk: int = 256, keep: tuple = ()) -> dict:
    """Whole-layer prefill forward (no KV cache), chunked over query rows.

    Returns a dict with ``out`` [B,L,d_model] plus any of ``q, k, v, var, k_values, scores,
    indices, mask, attn`` listed in ``keep`` (scores/indices/mask/attn are kept per chunk and
    concatenated, so only ask for them at small L).
    """
    B, L, _ = x.shape
    dtype = x.dtype
    if positions is None:
        positions = torch.arange(L).unsqueeze(0).expand(B, -1)
    if cos_cached is None:
        cos_cached, sin_cached = rope_cache(cfg.d_head, max(cfg.max_position_embeddings, L),
                                            cfg.rope_base, cfg.rope_scaling)
        cos_cached, sin_cached = cos_cached.to(dtype), sin_cached.to(dtype)
    q, k, v = project(W, cfg, x, positions, cos_cached, sin_cached)
    k_eff = k_effective(cfg, L)
    n_rep = cfg.n_heads // cfg.n_kv_heads
    scale = 1.0 / math.sqrt(cfg.d_head)

    # pass 1: per-row variance of every chunk (adaptive_topk.py:84-93)
    chunks = [(c, min(c + chunk, L)) for c in range(0, L, chunk)]
    var_parts, valid_parts, score_parts = [], [], []
    for c0, c1 in chunks:
        s = indexer_scores(W, x[:, c0:c1], x, cfg.n_indexer_heads, cfg.d_indexer,
                           cfg.indexer_activation, q_offset=c0)
        var_c, valid_c = row_variance(s)
        var_parts.append(var_c)
        valid_parts.append(valid_c)
        score_parts.append(s if "scores" in keep or L <= 4096 else None)
    var = torch.cat(var_parts, dim=1)
    valid = torch.cat(valid_parts, dim=1)
    if cfg.use_adaptive_k:
        k_values = adaptive_k(var, valid, var.mean(), cfg.k_base, cfg.k_min, cfg.k_max,
                              cfg.adaptive_k_temperature)
    else:
        k_values = torch.full((B, L), min(cfg.k_base, L), dtype=torch.long)

    # pass 2: selection and sparse attention per chunk
    attn_parts, idx_parts, mask_parts = [], [], []
    for (c0, c1), s in zip(chunks, score_parts):
        if s is None:
            s = indexer_scores(W, x[:, c0:c1], x, cfg.n_indexer_heads, cfg.d_indexer,
                               cfg.indexer_activation, q_offset=c0)
        idx, msk = topk_select(s, k_eff, k_values[:, c0:c1])
        a, _ = sparse_attention(q[:, c0:c1], k, v, idx, msk, n_rep, scale)
        attn_parts.append(a)
        if "indices" in keep:
            idx_parts.append(idx)
            mask_parts.append(msk)
    attn = torch.cat(attn_parts, dim=1)
    if cfg.use_output_gate:  # output_gate.py:101-126 (per_head=True)
        g = F.linear(x, W["output_gate.gate_proj.weight"], W["output_gate.gate_proj.bias"])
        gated = attn * gate_activation(g.view(B, L, cfg.n_heads, cfg.d_head), cfg.gate_activation)
    else:
        gated = attn
    out = F.linear(gated.reshape(B, L, -1), W["o_proj.weight"])  # gated_sparse_attention.py:229-230

    res = {"out": out}
    local = {"q": q, "k": k, "v": v, "var": var, "k_values": k_values, "attn": attn,
             "valid": valid}
    for name in keep:
        if name in local:
            res[name] = local[name]
    if "scores" in keep:
        res["scores"] = torch.cat(score_parts, dim=1)
    if "indices" in keep:
        res["indices"] = torch.cat(idx_parts, dim=1)
        res["mask"] = torch.cat(mask_parts, dim=1)
    return res


# --------------------------------------------------------------------------------------------
# Decoder layer and model  (gsa/models/gsa_llama.py)
# --------------------------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm.forward, gsa_llama.py:26-30."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).type_as(x) * weight


def swiglu_mlp(W: dict, prefix: str, x: torch.Tensor) -> torch.Tensor:
    """GSAMlp.forward, gsa_llama.py:45-46."""
    return F.linear(F.silu(F.linear(x, W[prefix + "gate_proj.weight"])) * F.linear(x, W[prefix + "up_proj.weight"]),
                    W[prefix + "down_proj.weight"])


def _sub(W: dict, prefix: str) -> dict:
    return {k[len(prefix):]: v for k, v in W.items() if k.startswith(prefix)}


def decoder_layer(W: dict, prefix: str, cfg: OracleConfig, eps: float, x: torch.Tensor, positions,
                  cos_cached, sin_cached, chunk: int = 256, keep: tuple = ()) -> dict:
    """GSADecoderLayer.forward without a cache, gsa_llama.py:93-112: x + GSA(norm(x)), then
    h + MLP(norm(h)).  Returns out plus the kept intermediates (normed, attn)."""
    normed = rms_norm(x, W[prefix + "input_layernorm.weight"], eps)
    attn = gsa_forward(_sub(W, prefix + "self_attn."), cfg, normed, positions, cos_cached, sin_cached,
                       chunk=chunk)["out"]
    h = x + attn
    out = h + swiglu_mlp(W, prefix + "mlp.", rms_norm(h, W[prefix + "post_attention_layernorm.weight"], eps))
    res = {"out": out}
    if "normed" in keep:
        res["normed"] = normed
    if "attn" in keep:
        res["attn"] = attn
    return res


def causal_lm_forward(W: dict, cfg: OracleConfig, n_layers: int, eps: float, input_ids: torch.Tensor,
                      cos_cached, sin_cached, chunk: int = 256, keep_layers: bool = False) -> dict:
    """GSALlamaForCausalLM.forward without labels or cache, gsa_llama.py:164-242 and 278-330:
    embedding, the decoder layers, the final norm and the LM head."""
    B, L = input_ids.shape
    positions = torch.arange(L).unsqueeze(0).expand(B, -1)
    h = F.embedding(input_ids, W["model.embed_tokens.weight"])
    res = {}
    for i in range(n_layers):
        r = decoder_layer(W, f"model.layers.{i}.", cfg, eps, h, positions, cos_cached, sin_cached, chunk,
                          keep=("normed", "attn") if keep_layers else ())
        h = r["out"]
        if keep_layers:
            res[f"layer{i}_normed"], res[f"layer{i}_attn"], res[f"layer{i}_out"] = r["normed"], r["attn"], h
    res["logits"] = F.linear(rms_norm(h, W["model.norm.weight"], eps), W["lm_head.weight"])
    return res

