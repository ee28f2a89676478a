"""GSA modules with the reference's API, computing through the sm_100a kernels.

Class names, constructor arguments, submodule and parameter names, buffers, return values and
error types follow the reference package ``gsa.attention`` (alfredcs/Gated-Sparse-Attention):

  GatedSparseAttention   gsa/attention/gated_sparse_attention.py:23-323
  GatedLightningIndexer  gsa/attention/gated_indexer.py:16-175
  AdaptiveTopKSelector   gsa/attention/adaptive_topk.py:14-211
  ValueGate              gsa/attention/value_gate.py:16-127
  OutputGate             gsa/attention/output_gate.py:15-142
  RotaryEmbedding        gsa/attention/rope.py:11-148
  apply_rotary_pos_emb   gsa/attention/rope.py:151-185

Submodules are created, and their weights initialised, in the reference's order, so
``torch.manual_seed(s); GatedSparseAttention(cfg)`` yields the same weights in both packages and
state dicts load either way.

The forward path of ``GatedSparseAttention`` is: one fused projection GEMM (cuBLAS), then the
library's kernels for RoPE / G2 / G1 gate / indexer weights, the chunked indexer + top-k
candidates, the adaptive k, the final selection, and the gathered sparse SDPA with the G1 gate
in its epilogue; ``o_proj`` is a cuBLAS GEMM.  No [B, L, L] score tensor and no gathered
[B, L, k, H, D] tensor is ever formed.  Inputs must be CUDA tensors in float32 or bfloat16;
there is no CPU path.

Steps that write into a KV cache (decode) append K, V and the indexer keys to a preallocated
store in place and run everything between the two GEMMs as one native call.  Under autograd the
prefill (no cache, unsharded) is differentiable: the backward runs the sparse-SDPA backward
kernel and cuBLAS GEMMs; the indexer gets no gradient, as in the reference.  Other autograd uses
raise ``NotImplementedError``.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from ._lib import ProjLayout

_ACTS = ("sigmoid", "tanh", "silu")


# ---------------------------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------------------------
class RotaryEmbedding(nn.Module):
    """RoPE tables (standard, NTK, YaRN).  Same buffers and arithmetic as rope.py:11-148."""

    def __init__(self, dim: int, max_position_embeddings: int = 131072, base: float = 10000.0,
                 scaling_config=None, device=None):
        super().__init__()
        self.dim = dim
        self.max_position_embeddings = max_position_embeddings
        self.base = base
        self.scaling_config = scaling_config or {}
        self.register_buffer("inv_freq", self._compute_inv_freq(device), persistent=False)
        self._set_cos_sin_cache(max_position_embeddings, device=device, dtype=torch.float32)

    def _compute_inv_freq(self, device=None) -> torch.Tensor:
        kind = self.scaling_config.get("type", None)
        ar = torch.arange(0, self.dim, 2, device=device).float()
        if kind == "yarn":  # rope.py:73-101
            factor = self.scaling_config.get("factor", 1.0)
            orig = self.scaling_config.get("original_max_position_embeddings", 4096)
            beta_fast = self.scaling_config.get("beta_fast", 32)
            beta_slow = self.scaling_config.get("beta_slow", 1)
            pos_freqs = self.base ** (ar / self.dim)
            extra = 1.0 / pos_freqs
            inter = 1.0 / (factor * pos_freqs)
            low = max(int(math.floor(self.dim * math.log(orig / (beta_fast * 2 * math.pi))
                                     / (2 * math.log(self.base)))), 0)
            high = min(int(math.ceil(self.dim * math.log(orig / (beta_slow * 2 * math.pi))
                                     / (2 * math.log(self.base)))), self.dim // 2 - 1)
            inv = inter.clone()
            inv[:low] = extra[:low]
            if high > low:
                smooth = (torch.arange(low, high + 1, device=device).float() - low) / (high - low)
                inv[low:high + 1] = (1 - smooth) * extra[low:high + 1] + smooth * inter[low:high + 1]
            return inv
        if kind == "ntk":  # rope.py:66-71
            factor = self.scaling_config.get("factor", 1.0)
            b = self.base * factor ** (self.dim / (self.dim - 2))
            return 1.0 / (b ** (ar / self.dim))
        # standard; "dynamic_ntk" uses the standard frequencies (rope.py:53-57)
        return 1.0 / (self.base ** (ar / self.dim))

    def _set_cos_sin_cache(self, seq_len: int, device=None, dtype=torch.float32):
        # rope.py:103-115, including its use of the cache dtype for the position ramp
        self.max_seq_len_cached = seq_len
        t = torch.arange(seq_len, device=device, dtype=dtype)
        freqs = torch.outer(t, self.inv_freq)
        emb = torch.cat((freqs, freqs), dim=-1)
        self.register_buffer("cos_cached", emb.cos(), persistent=False)
        self.register_buffer("sin_cached", emb.sin(), persistent=False)

    def ensure(self, seq_len: int):
        """Extend the tables to ``seq_len`` positions if needed (rope.py:136-142)."""
        if seq_len > self.max_seq_len_cached:
            self._set_cos_sin_cache(seq_len, device=self.cos_cached.device, dtype=self.cos_cached.dtype)

    def forward(self, positions: torch.Tensor, seq_len: Optional[int] = None):
        if seq_len is None:
            seq_len = int(positions.max().item()) + 1
        self.ensure(seq_len)
        return self.cos_cached[positions], self.sin_cached[positions]


def apply_rotary_pos_emb(q, k, cos, sin):
    """rotate-half RoPE on q [B,L,H,D] and k [B,L,Hk,D] (rope.py:151-185).  The attention layer
    applies RoPE inside its projection-epilogue kernel; this function is the standalone API."""
    cos = cos.unsqueeze(2)
    sin = sin.unsqueeze(2)

    def rot(x):
        h = x.shape[-1] // 2
        return x * cos + torch.cat([-x[..., h:], x[..., :h]], dim=-1) * sin

    return rot(q), rot(k)


# ---------------------------------------------------------------------------------------------
# Gates
# ---------------------------------------------------------------------------------------------
def _gate_stats(scores: Optional[torch.Tensor], per_head: bool = False) -> dict:
    if scores is None:
        return {}
    s = scores.float()
    out = {"mean": s.mean().item(), "std": s.std().item(), "min": s.min().item(),
           "max": s.max().item(), "sparsity": (s < 0.1).float().mean().item()}
    if per_head:
        out["per_head_mean"] = s.mean(dim=(0, 1, 3)).tolist() if s.dim() == 4 else None
    return out


def _gate_torch(logits: torch.Tensor, act: str) -> torch.Tensor:
    """act(logits) with the reference's torch ops, in the logits' dtype (value_gate.py:98-106)."""
    if act == "sigmoid":
        return torch.sigmoid(logits)
    if act == "tanh":
        return (torch.tanh(logits) + 1) / 2
    if act == "silu":
        return F.silu(logits)
    raise ValueError(f"Unknown activation: {act}")


class _LazyLogits:
    """A gate's logits h W^T + b, computed (torch GEMM) only if its scores are read: the fused
    projection kernel never writes them."""

    def __init__(self, x, weight, bias, shape):
        self.x, self.weight, self.bias, self.shape = x, weight, bias, shape

    def __call__(self) -> torch.Tensor:
        with torch.no_grad():
            return F.linear(self.x, self.weight, self.bias).view(self.shape)


class _GateScores:
    """``last_gate_scores`` of a gate module (value_gate.py:109-110, output_gate.py:122-123).  The
    fused attention layer does not run the gate modules: it hands each gate its logits (a view of
    the fused projection's output) and the activation is computed from them, with the reference's
    torch ops, when the scores are first read -- so the forward pays nothing for this analysis
    output.  Holding the view keeps the projection output alive until the scores are read or the
    next forward replaces them."""

    @property
    def last_gate_scores(self) -> Optional[torch.Tensor]:
        pending = self.__dict__.get("_pending_logits")
        if pending is not None:
            self.__dict__["_pending_logits"] = None
            if isinstance(pending, _LazyLogits):
                pending = pending()
            self.__dict__["_last_scores"] = _gate_torch(pending, self.activation).detach()
        return self.__dict__.get("_last_scores")

    @last_gate_scores.setter
    def last_gate_scores(self, value: Optional[torch.Tensor]):
        self.__dict__["_pending_logits"] = None
        self.__dict__["_last_scores"] = value

    def _set_pending_logits(self, logits: torch.Tensor):
        self.__dict__["_pending_logits"] = logits
        self.__dict__["_last_scores"] = None


class _GateFn(torch.autograd.Function):
    """out = x * act(logits) on the gate kernel.  The backward (the standalone gate modules under
    autograd; value_gate.py:95-113, output_gate.py:111-126) is fp32 elementwise:
    dx = dy * act(logits), dlogits = dy * x * act'(logits)."""

    @staticmethod
    def forward(ctx, x, logits, act, want_gate, holder):
        out, gate = ops.apply_gate(x, logits, act, want_gate=want_gate)
        holder.append(gate)
        ctx.act = act
        ctx.save_for_backward(x, logits)
        return out

    @staticmethod
    def backward(ctx, dy):
        x, logits = ctx.saved_tensors
        dyf = dy.float()
        dx = (dyf * _act(logits, ctx.act)).to(x.dtype) if ctx.needs_input_grad[0] else None
        dl = (dyf * x.float() * _act_grad(logits, ctx.act)).to(logits.dtype) if ctx.needs_input_grad[1] else None
        return dx, dl, None, None, None


def _gated(x: torch.Tensor, logits: torch.Tensor, act: str, want_gate: bool):
    """(x * act(logits), act(logits) or None): differentiable when autograd needs it."""
    if torch.is_grad_enabled() and (x.requires_grad or logits.requires_grad):
        holder = []
        out = _GateFn.apply(x, logits, act, want_gate, holder)
        return out, holder[0]
    return ops.apply_gate(x, logits, act, want_gate=want_gate)


class ValueGate(_GateScores, nn.Module):
    """G2: v * act(h W^T + b) per KV-head element (value_gate.py:16-127)."""

    def __init__(self, d_model: int, n_kv_heads: int, d_head: int, bias_init: float = 0.5,
                 activation: str = "sigmoid"):
        super().__init__()
        self.d_model = d_model
        self.n_kv_heads = n_kv_heads
        self.d_head = d_head
        self.activation = activation
        self.gate_proj = nn.Linear(d_model, n_kv_heads * d_head, bias=True)
        self._init_weights(bias_init)
        self.last_gate_scores: Optional[torch.Tensor] = None

    def _init_weights(self, bias_init: float):
        nn.init.xavier_uniform_(self.gate_proj.weight, gain=0.1)
        nn.init.constant_(self.gate_proj.bias, bias_init)

    def forward(self, v: torch.Tensor, hidden_states: torch.Tensor) -> torch.Tensor:
        if self.activation not in _ACTS:
            raise ValueError(f"Unknown activation: {self.activation}")
        logits = self.gate_proj(hidden_states).view_as(v)
        out, gate = _gated(v, logits, self.activation, not self.training)
        if not self.training:
            self.last_gate_scores = gate.detach()
        return out

    def get_gate_statistics(self) -> dict:
        return _gate_stats(self.last_gate_scores)


class OutputGate(_GateScores, nn.Module):
    """G1: o * act(h W^T + b), per head element or per head scalar (output_gate.py:15-142)."""

    def __init__(self, d_model: int, n_heads: int, d_head: int, bias_init: float = 0.5,
                 activation: str = "sigmoid", per_head: bool = True):
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.d_head = d_head
        self.activation = activation
        self.per_head = per_head
        out = n_heads * d_head if per_head else n_heads
        self.gate_proj = nn.Linear(d_model, out, bias=True)
        self._init_weights(bias_init)
        self.last_gate_scores: Optional[torch.Tensor] = None

    def _init_weights(self, bias_init: float):
        nn.init.xavier_uniform_(self.gate_proj.weight, gain=0.1)
        nn.init.constant_(self.gate_proj.bias, bias_init)

    def forward(self, attn_output: torch.Tensor, hidden_states: torch.Tensor) -> torch.Tensor:
        if self.activation not in _ACTS:
            raise ValueError(f"Unknown activation: {self.activation}")
        B, L, H, D = attn_output.shape
        logits = self.gate_proj(hidden_states)
        logits = logits.view(B, L, H, D) if self.per_head else logits.view(B, L, H, 1).expand(B, L, H, D)
        out, gate = _gated(attn_output, logits, self.activation, not self.training)
        if not self.training:
            self.last_gate_scores = (gate if self.per_head else gate[..., :1]).detach()
        return out

    def get_gate_statistics(self) -> dict:
        return _gate_stats(self.last_gate_scores, per_head=True)


# ---------------------------------------------------------------------------------------------
# Indexer and selector
# ---------------------------------------------------------------------------------------------
class _IndexerScoresFn(torch.autograd.Function):
    """Indexer scores on the indexer kernel (gated_indexer.py:123-153).  The backward (the standalone
    indexer module under autograd) recomputes the pre-activations z = scale q^I.k^I + b in fp32 and
    returns, with dI the incoming gradient (zero at masked entries, as masked_fill makes it):
      dz = dI * w_j * act'(z); dw_j = sum_s dI * act(z); dq^I = scale dz k^I; dk^I = scale sum_j dz q^I_j;
      db_j = sum dz."""

    @staticmethod
    def forward(ctx, q_idx, k_idx, w, bias, dims, scale, causal, act):
        scores = ops.indexer_scores(dims, q_idx, k_idx, w, bias, scale, q_pos0=0, causal=causal)
        ctx.save_for_backward(q_idx, k_idx, w, bias)
        ctx.meta = (dims.n_idx_heads, dims.d_idx, scale, causal, act)
        return scores

    @staticmethod
    def backward(ctx, d_scores):
        q_idx, k_idx, w, bias = ctx.saved_tensors
        HI, dI, scale, causal, act = ctx.meta
        B, Lq, _ = q_idx.shape
        Lkv = k_idx.shape[1]
        q = q_idx.float().reshape(B, Lq, HI, dI)
        k = k_idx.float()
        g = d_scores.float()
        if causal:
            fut = torch.ones(Lq, Lkv, dtype=torch.bool, device=g.device).triu(1)
            g = g.masked_fill(fut, 0.0)
        z = torch.einsum("bqhd,bkd->bhqk", q, k) * scale + bias.float().view(1, -1, 1, 1)
        if act == "sigmoid":
            a = torch.sigmoid(z)
            da = a * (1 - a)
        else:
            a = F.relu(z)
            da = (z > 0).float()
        wt = w.float().permute(0, 2, 1).unsqueeze(-1)               # [B, HI, Lq, 1]
        dz = g.unsqueeze(1) * wt * da                               # [B, HI, Lq, Lkv]
        dw = (g.unsqueeze(1) * a).sum(-1).permute(0, 2, 1)          # [B, Lq, HI]
        dq = (torch.einsum("bhqk,bkd->bqhd", dz, k) * scale).reshape(B, Lq, HI * dI)
        dk = torch.einsum("bhqk,bqhd->bkd", dz, q) * scale
        db = dz.sum(dim=(0, 2, 3))
        return dq.to(q_idx.dtype), dk.to(k_idx.dtype), dw.to(w.dtype), db.to(bias.dtype), None, None, None, None


class GatedLightningIndexer(nn.Module):
    """I[t,s] = sum_j sigmoid(h_t W_j^Iw) * act(q^I_{t,j} . k^I_s / sqrt(d_I) + b_j)
    (gated_indexer.py:16-175).  ``forward`` materialises [B, Lq, Lkv] scores for callers that
    want them; the attention layer never does."""

    def __init__(self, d_model: int, d_indexer: int = 64, n_indexer_heads: int = 4,
                 activation: str = "sigmoid", use_causal_mask: bool = True):
        super().__init__()
        self.d_model = d_model
        self.d_indexer = d_indexer
        self.n_indexer_heads = n_indexer_heads
        self.activation = activation
        self.use_causal_mask = use_causal_mask
        self.q_proj = nn.Linear(d_model, n_indexer_heads * d_indexer, bias=False)
        self.k_proj = nn.Linear(d_model, d_indexer, bias=False)
        self.weight_proj = nn.Linear(d_model, n_indexer_heads, bias=True)
        self.bias = nn.Parameter(torch.zeros(n_indexer_heads))
        self.scale = 1.0 / math.sqrt(d_indexer)
        self._init_weights()

    def _init_weights(self):
        nn.init.xavier_uniform_(self.q_proj.weight, gain=1.0)
        nn.init.xavier_uniform_(self.k_proj.weight, gain=1.0)
        nn.init.xavier_uniform_(self.weight_proj.weight, gain=0.1)
        nn.init.zeros_(self.weight_proj.bias)
        nn.init.zeros_(self.bias)

    def _dims(self):
        return ops.make_dims(self.d_model, 1, 1, 2, self.n_indexer_heads, self.d_indexer,
                             "sigmoid", self.activation)

    def forward(self, hidden_states: torch.Tensor, positions: Optional[torch.Tensor] = None,
                kv_hidden_states: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.activation not in ("sigmoid", "relu"):
            raise ValueError(f"Unknown activation: {self.activation}")
        if kv_hidden_states is None:
            kv_hidden_states = hidden_states
        B, Lq, _ = hidden_states.shape
        Lkv = kv_hidden_states.shape[1]
        causal = self.use_causal_mask and Lq == Lkv
        q_idx = F.linear(hidden_states, self.q_proj.weight)
        k_idx = F.linear(kv_hidden_states, self.k_proj.weight)
        w = torch.sigmoid(self.weight_proj(hidden_states))
        if torch.is_grad_enabled() and any(t.requires_grad for t in (q_idx, k_idx, w, self.bias)):
            scores = _IndexerScoresFn.apply(q_idx, k_idx, w, self.bias, self._dims(), self.scale, causal,
                                            self.activation)
        else:
            scores = ops.indexer_scores(self._dims(), q_idx, k_idx, w, self.bias, self.scale, q_pos0=0,
                                        causal=causal)
        return scores.to(hidden_states.dtype)

    def get_indexer_statistics(self, hidden_states: torch.Tensor) -> dict:
        with torch.no_grad():
            scores = self.forward(hidden_states)
            valid = scores[scores != float("-inf")].float()
            return {"mean": valid.mean().item(), "std": valid.std().item(),
                    "min": valid.min().item(), "max": valid.max().item(),
                    "sparsity": (valid < 0.1).float().mean().item(),
                    "head_weights": torch.sigmoid(self.weight_proj.bias).tolist()}


class AdaptiveTopKSelector(nn.Module):
    """Per-row k_t from the score variance and the top-k_t selection (adaptive_topk.py:14-211).

    Returns ``(indices, mask)`` [B, Lq, k_eff]: ``indices`` holds the k_eff best columns of each
    row in ascending column order and ``mask`` marks the k_t of them that are kept.  The
    reference returns the same candidate columns sorted by score; every consumer uses the
    (indices, mask) pair as a set, so the two are interchangeable."""

    def __init__(self, k_base: int = 2048, k_min: int = 256, k_max: int = 4096,
                 use_adaptive: bool = True, temperature: float = 1.0,
                 adaptive_method: str = "variance"):
        super().__init__()
        self.k_base = k_base
        self.k_min = k_min
        self.k_max = k_max
        self.use_adaptive = use_adaptive
        self.temperature = temperature
        self.adaptive_method = adaptive_method
        if adaptive_method == "learned":  # [mean, std, max] of a row's scores -> fraction of [k_min, k_max]
            self.k_predictor = nn.Sequential(nn.Linear(3, 32), nn.ReLU(), nn.Linear(32, 1), nn.Sigmoid())

    def _k_from_summary(self, s2d: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """k_t of the entropy and learned methods (adaptive_topk.py:104-133): the row statistics
        come from the native row-summary pass; the few per-row scalar ops follow on them (the
        learned method through the module's own predictor)."""
        summ = ops.row_summary(s2d, dtype)
        valid = summ[:, 0]
        if self.adaptive_method == "entropy":
            # the entropy is a dtype value; the division promotes it to fp32
            norm = summ[:, 4] / (torch.log(valid + 1) + 1e-8)
            k_adaptive = self.k_base * (0.5 + norm * self.temperature)
        else:
            stats = summ[:, 1:4].to(dtype)
            k_scale = self.k_predictor(stats).squeeze(-1)
            k_adaptive = self.k_min + k_scale * (self.k_max - self.k_min)
        k = torch.minimum(torch.clamp(k_adaptive, self.k_min, self.k_max), valid)
        return k.long().to(torch.int32)

    def forward(self, scores: torch.Tensor, seq_q: int, seq_kv: int, return_k_values: bool = False):
        B, Lq, Lkv = scores.shape
        if self.use_adaptive and self.adaptive_method not in ("variance", "entropy", "learned"):
            raise ValueError(f"Unknown adaptive method: {self.adaptive_method}")
        k_eff = min(self.k_max, seq_kv) if self.use_adaptive else min(self.k_base, seq_kv)
        s2d = scores.reshape(B * Lq, Lkv).float()
        cand_idx, cand_score, cand_count = ops.topk_candidates(s2d, k_eff)
        if self.use_adaptive and self.adaptive_method != "variance":
            k = self._k_from_summary(s2d, scores.dtype)
        elif self.use_adaptive:
            stats = ops.row_stats(s2d)
            var, total = ops.row_variance(stats, Lkv, scores.dtype)
            k = ops.adaptive_k(stats, var, total, Lkv, scores.dtype, self.k_base, self.k_min,
                               self.k_max, True, self.temperature)
        else:
            k = torch.full((B * Lq,), min(self.k_base, seq_kv), device=scores.device, dtype=torch.int32)
        _, _, mask = ops.select_finalize(cand_idx, cand_score, cand_count, k, want_mask=True)
        indices = cand_idx.long().view(B, Lq, k_eff)
        mask = mask.bool().view(B, Lq, k_eff)
        if return_k_values:
            return indices, mask, k.long().view(B, Lq)
        return indices, mask

    def get_selection_statistics(self, scores: torch.Tensor) -> dict:
        with torch.no_grad():
            _, mask, k_values = self.forward(scores, scores.shape[1], scores.shape[2], return_k_values=True)
            return {"k_mean": k_values.float().mean().item(), "k_std": k_values.float().std().item(),
                    "k_min": k_values.min().item(), "k_max": k_values.max().item(),
                    "coverage": mask.float().mean().item()}


# ---------------------------------------------------------------------------------------------
# KV cache
# ---------------------------------------------------------------------------------------------
class KVCacheStore:
    """Preallocated buffers of one layer's KV cache: K and V interleaved per token
    [B, capacity, 2, Hk, D] (the layout the sparse SDPA reads) and the indexer keys
    [B, capacity, d_I].  ``filled`` is the number of leading tokens some cache handed out holds;
    a cache of exactly that length may append in place, any other length copies first, so that
    two continuations of one cache never write the same slots.  The store also keeps the
    scratch of the native step (sized for its capacity), so that a decode loop allocates
    nothing per step."""

    def __init__(self, batch: int, capacity: int, n_kv_heads: int, d_head: int, d_idx: int,
                 dtype: torch.dtype, device):
        self.kv = torch.empty(batch, capacity, 2, n_kv_heads, d_head, dtype=dtype, device=device)
        self.ki = torch.empty(batch, capacity, d_idx, dtype=dtype, device=device)
        self.filled = 0
        self._scratch = {}

    def scratch(self, key, nbytes: int) -> torch.Tensor:
        t = self._scratch.get(key)
        if t is None or t.numel() < nbytes:
            t = torch.empty(nbytes, dtype=torch.uint8, device=self.kv.device)
            self._scratch[key] = t
        return t

    @property
    def capacity(self) -> int:
        return self.kv.shape[1]

    def fits(self, batch: int, length: int, dtype, device) -> bool:
        return (self.kv.shape[0] == batch and length <= self.capacity and self.kv.dtype == dtype
                and self.kv.device == device)

    def view(self, n: int) -> "GSAKVCache":
        kv = self.kv[:, :n]
        return GSAKVCache(kv[:, :, 0], kv[:, :, 1], self.ki[:, :n], kv, self)


def _grown_capacity(n: int) -> int:
    """Capacity of a new cache store for n tokens: a quarter (at least 256 tokens) of headroom,
    rounded up to 256, so that a decode loop reallocates O(log) times."""
    return (n + max(n // 4, 256) + 255) // 256 * 256


class GSAKVCache(tuple):
    """The (k, v) cache pair of the reference (post-RoPE k, post-G2 v, [B, Lkv, Hk, D]) that
    also carries the indexer keys k^I [B, Lkv, d_I].  It is a 2-tuple, so code written for the
    reference's cache keeps working; when it is passed back as ``past_key_value`` the indexer
    scores the new queries against every cached key.

    A cache returned by the layer is a view of a :class:`KVCacheStore` with room for more
    tokens: passing it back appends the new tokens' K, V and k^I in place (the reference
    concatenates the whole cache every step, gated_sparse_attention.py:188-192); when the store
    is full, or when this cache is not the longest view of its store, the layer moves to a new,
    larger store first.  ``GatedSparseAttention.allocate_cache`` preallocates one."""

    def __new__(cls, k, v, indexer_keys=None, kv=None, store=None):
        obj = super().__new__(cls, (k, v))
        obj.indexer_keys = indexer_keys
        obj.kv = kv  # the interleaved [B, Lkv, 2, Hk, D] buffer k and v are views of
        obj.store = store
        return obj

    @property
    def capacity(self) -> int:
        """Tokens this cache can hold before the layer moves it to a larger store."""
        return self.store.capacity if self.store is not None else self[0].shape[1]


class _ForwardOnly(torch.autograd.Function):
    @staticmethod
    def forward(ctx, out, *_):
        return out.view_as(out)

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError("the B200 GSA layer's backward covers the prefill without a KV cache, "
                                  "unsharded, without output_attentions")


def _act(logits: torch.Tensor, act: str) -> torch.Tensor:
    """The gate activations in fp32 (value_gate.py:98-106: tanh is rescaled to (0, 1))."""
    x = logits.float()
    if act == "sigmoid":
        return torch.sigmoid(x)
    if act == "tanh":
        return (torch.tanh(x) + 1) / 2
    if act == "silu":
        return F.silu(x)
    raise ValueError(f"Unknown activation: {act}")


def _act_grad(logits: torch.Tensor, act: str) -> torch.Tensor:
    """d act(x) / dx in fp32 for the gate activations (value_gate.py:98-106, output_gate.py:111-119)."""
    x = logits.float()
    if act == "sigmoid":
        g = torch.sigmoid(x)
        return g * (1 - g)
    if act == "tanh":
        return (1 - torch.tanh(x) ** 2) / 2
    if act == "silu":
        g = torch.sigmoid(x)
        return g * (1 + x * (1 - g))
    raise ValueError(f"Unknown activation: {act}")


def _rope_backward(dy: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Transpose of y = x cos + rotate_half(x) sin (rope.py:151-185): rotate_half maps (x1, x2) to
    (-x2, x1), its transpose maps (y1, y2) to (y2, -y1).  dy [T, heads, D] fp32, cos/sin [T, D]."""
    c, s_ = cos.float().unsqueeze(1), sin.float().unsqueeze(1)
    ys = dy * s_
    h = dy.shape[-1] // 2
    return dy * c + torch.cat([ys[..., h:], -ys[..., :h]], dim=-1)


class _GSATrain(torch.autograd.Function):
    """The layer's forward on the B200 kernels with the backward of the differentiable part:
    o_proj, the G1 gate, the sparse SDPA over the selected keys (gsa_sparse_sdpa_backward), RoPE,
    the G2 gate and the fused q/k/v/gate projections.  The selection (torch.topk indices,
    adaptive_topk.py:177) carries no gradient, so neither does the indexer -- as in the
    reference, whose only path from the indexer to the output is through those indices."""

    @staticmethod
    def forward(ctx, layer, x, W, bvec, Wo, positions):
        with torch.no_grad():
            saved = {}
            out, _, _ = layer._forward_impl(x, positions, None, False, False, train=saved)
        ctx.layer = layer
        ctx.saved = saved
        ctx.save_for_backward(x, W, Wo)
        return out

    @staticmethod
    def backward(ctx, d_out):
        layer, sv = ctx.layer, ctx.saved
        x, W, Wo = ctx.saved_tensors
        B, L, dm = x.shape
        H, Hk, D = layer.n_heads, layer.n_kv_heads, layer.d_head
        T = B * L
        lay = sv["layout"]
        with torch.no_grad():
            # GEMMs in the parameters' dtype (tensor cores for bf16, fp32 accumulation), as torch
            # autograd runs them; the elementwise parts in fp32
            dt = Wo.dtype
            dout = d_out.reshape(T, dm).to(dt)
            gated = sv["gated"].reshape(T, H * D)
            dWo = dout.t() @ gated
            d_gated = (dout @ Wo).view(T, H, D).float()
            O, g1 = sv["O"].view(T, H, D), sv["g1"]
            proj = sv["proj"]
            if g1 is not None:
                g1 = g1.view(T, H, D)
                dO = d_gated * g1.float()
                act = layer.output_gate.activation
                d_g1 = (d_gated * O.float()) * _act_grad(proj[:, lay.g1:lay.g1 + H * D].view(T, H, D), act)
            else:
                dO, d_g1 = d_gated, None
            dq, dk, dv = ops.sparse_sdpa_backward(sv["dims"], sv["q"], sv["k"], sv["v"], sv["sel"], sv["cnt"],
                                                  sv["O"], dO.view(B, L, H, D), sv["lse"], layer.scale)
            pos = sv["positions"].reshape(-1)
            cos, sin = layer.rotary_emb.cos_cached[pos], layer.rotary_emb.sin_cached[pos]
            dq_raw = _rope_backward(dq.view(T, H, D), cos, sin)
            dk_raw = _rope_backward(dk.reshape(T, Hk, D), cos, sin)
            dv = dv.reshape(T, Hk * D)
            d_proj = torch.zeros(T, W.shape[0], device=x.device, dtype=torch.float32)
            d_proj[:, lay.q:lay.q + H * D] = dq_raw.reshape(T, H * D)
            d_proj[:, lay.k:lay.k + Hk * D] = dk_raw.reshape(T, Hk * D)
            if lay.g2 >= 0:
                act = layer.value_gate.activation
                v_raw = proj[:, lay.v:lay.v + Hk * D].float()
                g2l = proj[:, lay.g2:lay.g2 + Hk * D]
                g2 = _act(g2l, act)
                d_proj[:, lay.v:lay.v + Hk * D] = dv * g2
                d_proj[:, lay.g2:lay.g2 + Hk * D] = dv * v_raw * _act_grad(g2l, act)
            else:
                d_proj[:, lay.v:lay.v + Hk * D] = dv
            if d_g1 is not None:
                d_proj[:, lay.g1:lay.g1 + H * D] = d_g1.reshape(T, H * D)
            x2 = x.reshape(T, dm)
            db = d_proj.sum(0).to(W.dtype) if ctx.needs_input_grad[3] else None
            d_proj = d_proj.to(W.dtype)
            dx = (d_proj @ W).to(x.dtype).view(B, L, dm) if ctx.needs_input_grad[1] else None
            dW = d_proj.t() @ x2.to(W.dtype) if ctx.needs_input_grad[2] else None
        return None, dx, dW, db, (dWo if ctx.needs_input_grad[4] else None), None


# ---------------------------------------------------------------------------------------------
# The layer
# ---------------------------------------------------------------------------------------------
class GatedSparseAttention(nn.Module):
    """Gated Sparse Attention layer (gated_sparse_attention.py:23-323), forward on sm_100a."""

    def __init__(self, config):
        super().__init__()
        self.config = config
        self.d_model = config.d_model
        self.n_heads = config.n_heads
        self.n_kv_heads = config.n_kv_heads
        self.d_head = config.d_head
        self.n_rep = self.n_heads // self.n_kv_heads
        self.scale = 1.0 / math.sqrt(self.d_head)
        # candidate pass: "auto" takes the threshold-survivor pass where it applies (sigmoid
        # indexer), "exact" always selects each row's k_eff best first; the keys finally
        # selected are the same
        self.selection_path = "auto"

        self.q_proj = nn.Linear(self.d_model, self.n_heads * self.d_head, bias=False)
        self.k_proj = nn.Linear(self.d_model, self.n_kv_heads * self.d_head, bias=False)
        self.v_proj = nn.Linear(self.d_model, self.n_kv_heads * self.d_head, bias=False)
        self.o_proj = nn.Linear(self.n_heads * self.d_head, self.d_model, bias=False)
        self.indexer = GatedLightningIndexer(d_model=self.d_model, d_indexer=config.d_indexer,
                                             n_indexer_heads=config.n_indexer_heads,
                                             activation=config.indexer_activation)
        self.topk_selector = AdaptiveTopKSelector(k_base=config.k_base, k_min=config.k_min,
                                                  k_max=config.k_max, use_adaptive=config.use_adaptive_k,
                                                  temperature=config.adaptive_k_temperature)
        self.value_gate = (ValueGate(self.d_model, self.n_kv_heads, self.d_head, bias_init=config.gate_bias_init)
                           if config.use_value_gate else None)
        self.output_gate = (OutputGate(self.d_model, self.n_heads, self.d_head, bias_init=config.gate_bias_init)
                            if config.use_output_gate else None)
        self.rotary_emb = RotaryEmbedding(dim=self.d_head, max_position_embeddings=config.max_position_embeddings,
                                          base=config.rope_base, scaling_config=config.rope_scaling)
        self.attn_dropout = nn.Dropout(config.attention_dropout)
        self.dense_residual_alpha = config.dense_residual_alpha
        self._init_weights()
        self._fused = None
        # set by gsa_b200.sharded.enable_query_sharding: this rank's share of the query sequence
        self.query_shards = None
        # set by gsa_b200.sharded.enable_sequence_sharding: the process group whose ranks hold
        # the other sequences of the batch (the adaptive k's variance mean spans them)
        self.sequence_shards = None
        # steps that write into a KV cache store run everything between the two GEMMs as one
        # native call (gsa_decode_attend); False runs the same kernels one by one from Python
        self.native_step = True
        self._static = None
        # bf16 prefill: one tensor-core GEMM with the projection epilogue fused (when the shapes allow
        # it: both gates, d_head 64 or 128, ...); False runs cuBLAS and the separate epilogue kernel
        self.fused_gemm = True
        self._fused_tiles = None

    def allocate_cache(self, batch_size: int, capacity: int, dtype: Optional[torch.dtype] = None,
                       device=None) -> "GSAKVCache":
        """An empty KV cache (length 0) with room for ``capacity`` tokens of each of
        ``batch_size`` sequences.  Pass it as ``past_key_value`` of the prefill (with
        ``use_cache=True``); the prefill and every decode step then write K, V and the indexer
        keys into it in place."""
        w = self.q_proj.weight
        store = KVCacheStore(batch_size, capacity, self.n_kv_heads, self.d_head, self.config.d_indexer,
                             dtype or w.dtype, device or w.device)
        return store.view(0)

    def _init_weights(self):
        for module in [self.q_proj, self.k_proj, self.v_proj]:
            nn.init.xavier_uniform_(module.weight, gain=1.0 / math.sqrt(2))
        nn.init.xavier_uniform_(self.o_proj.weight, gain=1.0 / math.sqrt(2 * self.config.n_layers))

    def _repeat_kv(self, x: torch.Tensor) -> torch.Tensor:
        """[B, L, Hk, D] -> [B, L, H, D] (gated_sparse_attention.py:123-137)."""
        B, L, Hk, D = x.shape
        if self.n_rep == 1:
            return x
        return x.unsqueeze(3).expand(B, L, Hk, self.n_rep, D).reshape(B, L, self.n_heads, D)

    # -- fused projection weight ------------------------------------------------------------
    def _segments(self):
        H, Hk, D = self.n_heads, self.n_kv_heads, self.d_head
        ix = self.indexer
        segs = [("q", self.q_proj.weight, None), ("k", self.k_proj.weight, None),
                ("v", self.v_proj.weight, None)]
        if self.value_gate is not None:
            segs.append(("g2", self.value_gate.gate_proj.weight, self.value_gate.gate_proj.bias))
        if self.output_gate is not None:
            if not self.output_gate.per_head:
                raise NotImplementedError("the fused layer supports the per-head output gate only")
            segs.append(("g1", self.output_gate.gate_proj.weight, self.output_gate.gate_proj.bias))
        segs += [("qi", ix.q_proj.weight, None), ("ki", ix.k_proj.weight, None),
                 ("wi", ix.weight_proj.weight, ix.weight_proj.bias)]
        return segs

    def fused_projection(self):
        """(W [Ncat, d_model], b [Ncat], ProjLayout): every projection of the layer stacked so
        that one GEMM produces all of them; Ncat is padded to a multiple of 64.  Cached until a
        parameter changes."""
        segs = self._segments()
        key = tuple((n, w.data_ptr(), w._version, None if b is None else (b.data_ptr(), b._version))
                    for n, w, b in segs)
        if self._fused is not None and self._fused[0] == key:
            return self._fused[1:]
        ws, bs, offs, off = [], [], {}, 0
        for name, w, b in segs:
            offs[name] = off
            ws.append(w.detach())
            bs.append(b.detach() if b is not None else torch.zeros(w.shape[0], device=w.device, dtype=w.dtype))
            off += w.shape[0]
        pad = (-off) % 64
        if pad:
            ws.append(torch.zeros(pad, self.d_model, device=ws[0].device, dtype=ws[0].dtype))
            bs.append(torch.zeros(pad, device=ws[0].device, dtype=ws[0].dtype))
        W = torch.cat(ws, 0).contiguous()
        bvec = torch.cat(bs, 0).contiguous()
        layout = ProjLayout(*(offs.get(n, -1) for n in ("q", "k", "v", "g2", "g1", "qi", "ki", "wi")))
        self._fused = (key, W, bvec, layout)
        return W, bvec, layout

    def fused_projection_tiles(self):
        """(Wp [rows, d_model], bias [rows] fp32): the projection weights and biases in the row order of
        the fused projection GEMM -- q, k, then v_h and g2_h head by head, g1, q^I, k^I, w, zero rows
        to gsa_proj_fused_rows -- cached until a parameter changes."""
        segs = self._segments()
        key = tuple((n, w.data_ptr(), w._version, None if b is None else (b.data_ptr(), b._version))
                    for n, w, b in segs)
        if self._fused_tiles is not None and self._fused_tiles[0] == key:
            return self._fused_tiles[1:]
        by = {n: (w.detach(), None if b is None else b.detach()) for n, w, b in segs}
        H, Hk, D = self.n_heads, self.n_kv_heads, self.d_head
        ws, bs = [], []

        def add(w, b):
            ws.append(w)
            bs.append(torch.zeros(w.shape[0], device=w.device, dtype=torch.float32) if b is None else b.float())

        add(*by["q"])
        add(*by["k"])
        vw, g2w, g2b = by["v"][0], by["g2"][0], by["g2"][1]
        for h in range(Hk):
            add(vw[h * D:(h + 1) * D], None)
            add(g2w[h * D:(h + 1) * D], g2b[h * D:(h + 1) * D])
        add(*by["g1"])
        add(*by["qi"])
        add(*by["ki"])
        add(*by["wi"])
        rows = ops.proj_fused_rows(self._dims())
        n = sum(w.shape[0] for w in ws)
        if rows > n:
            ws.append(torch.zeros(rows - n, self.d_model, device=ws[0].device, dtype=ws[0].dtype))
            bs.append(torch.zeros(rows - n, device=ws[0].device, dtype=torch.float32))
        Wp = torch.cat(ws, 0).contiguous()
        bp = torch.cat(bs, 0).contiguous()
        self._fused_tiles = (key, Wp, bp)
        return Wp, bp

    def _dims(self):
        return ops.make_dims(self.d_model, self.n_heads, self.n_kv_heads, self.d_head,
                             self.config.n_indexer_heads, self.config.d_indexer,
                             self.value_gate.activation if self.value_gate is not None else
                             (self.output_gate.activation if self.output_gate is not None else "sigmoid"),
                             self.indexer.activation)

    def _step_constants(self):
        """(dims, top-k parameters, fp32 indexer bias) of the native step, rebuilt when the
        indexer bias changes."""
        b = self.indexer.bias
        key = (b.data_ptr(), b._version, b.dtype)
        if self._static is None or self._static[0] != key:
            cfg = self.config
            tp = ops.TopkParams(cfg.k_base, cfg.k_min, cfg.k_max, int(cfg.use_adaptive_k),
                                float(cfg.adaptive_k_temperature))
            self._static = (key, self._dims(), tp, b.detach().float().contiguous())
        return self._static[1:]

    # -- forward ----------------------------------------------------------------------------
    def forward(self, hidden_states: torch.Tensor, positions: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                past_key_value: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                use_cache: bool = False, output_attentions: bool = False):
        x = hidden_states
        if not x.is_cuda:
            raise RuntimeError("GatedSparseAttention (B200) runs on CUDA tensors only")
        if self.training and self.attn_dropout.p > 0:
            raise NotImplementedError("attention dropout in training mode is not implemented")
        if (self.value_gate is not None and self.output_gate is not None
                and self.value_gate.activation != self.output_gate.activation):
            raise NotImplementedError("value and output gates must share one activation")
        params = [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self.o_proj.weight]
        for gate in (self.value_gate, self.output_gate):
            if gate is not None:
                params += [gate.gate_proj.weight, gate.gate_proj.bias]
        needs_grad = torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in params))
        if (needs_grad and past_key_value is None and not use_cache and not output_attentions
                and self.query_shards is None and self.sequence_shards is None):
            W, bvec = self._train_projection()
            out = _GSATrain.apply(self, x, W, bvec, self.o_proj.weight, positions)
            return out, None, None
        with torch.no_grad():
            out, present, weights = self._forward_impl(x, positions, past_key_value, use_cache,
                                                       output_attentions)
        if needs_grad:
            out = _ForwardOnly.apply(out, x, self.q_proj.weight)
        return out, present, weights if output_attentions else None

    def _train_projection(self):
        """The fused projection weight and bias built inside the autograd graph: gradients reach
        q/k/v and the gate projections; the indexer's segments are detached (no gradient, as in
        the reference)."""
        ws, bs = [], []
        for name, w, b in self._segments():
            diff = name in ("q", "k", "v", "g2", "g1")
            ws.append(w if diff else w.detach())
            if b is None:
                bs.append(torch.zeros(w.shape[0], device=w.device, dtype=w.dtype))
            else:
                bs.append(b if diff else b.detach())
        n = sum(w.shape[0] for w in ws)
        pad = (-n) % 64
        if pad:
            ws.append(torch.zeros(pad, self.d_model, device=ws[0].device, dtype=ws[0].dtype))
            bs.append(torch.zeros(pad, device=ws[0].device, dtype=ws[0].dtype))
        return torch.cat(ws, 0), torch.cat(bs, 0)

    def _forward_impl(self, x, positions, past_key_value, use_cache, output_attentions,
                      mark=None, capture=None, train=None):
        """The forward computation.  ``mark(name)`` (optional) is called after each stage and
        ``capture`` (optional dict) receives the SDPA inputs; both are for measurement (and
        keep the stages apart, one call each)."""
        mark_fn = mark
        mark = mark or (lambda name: None)
        B, L, _ = x.shape
        dt = x.dtype
        ops.dtype_code(dt)
        H, Hk, D = self.n_heads, self.n_kv_heads, self.d_head
        HI, dI = self.config.n_indexer_heads, self.config.d_indexer
        cfg = self.config
        sp = self.query_shards
        if sp is not None and past_key_value is not None:
            raise NotImplementedError("query-sharded layers run prefill without a KV cache")
        past_len = past_key_value[0].shape[1] if past_key_value is not None else 0
        # (local row start, rows, absolute position of the first row) of each query segment
        segs = sp.segments(L) if sp is not None else [(0, L, past_len)]
        if sp is not None and len(segs) > 1 and B != 1:
            raise NotImplementedError("zigzag query sharding takes one sequence per call")
        positions_given = positions is not None
        if positions is None:
            max_pos = max(p0 + n - 1 for _, n, p0 in segs)
        else:
            max_pos = int(positions.max().item())  # the reference syncs here too (rope.py:133-134)
        self.rotary_emb.ensure(max_pos + 1)
        if self.q_proj.weight.dtype != dt:
            raise RuntimeError(f"layer parameters are {self.q_proj.weight.dtype} but the input is {dt}")
        dims = self._step_constants()[0]

        # the KV cache store the new tokens' K, V and k^I are written into (None: a fresh
        # [B, L, 2, Hk, D] buffer), and whether the returned cache may claim them
        store = None
        if sp is None and (past_key_value is None or getattr(past_key_value, "indexer_keys", None) is not None):
            old = getattr(past_key_value, "store", None) if past_key_value is not None else None
            if old is not None and old.filled == past_len and old.fits(B, past_len + L, dt, x.device):
                store = old
            elif past_key_value is not None or use_cache:
                store = KVCacheStore(B, _grown_capacity(past_len + L), Hk, D, dI, dt, x.device)
                if past_len:
                    store.kv[:, :past_len, 0] = past_key_value[0]
                    store.kv[:, :past_len, 1] = past_key_value[1]
                    store.ki[:, :past_len] = past_key_value.indexer_keys
                store.filled = past_len

        n_all = past_len + L
        native = (store is not None and self.native_step and self.selection_path == "auto" and mark_fn is None
                  and capture is None and not output_attentions
                  and B * L * ((n_all + 3) // 4 * 4) * 4 <= ops.SCORE_CHUNK_BYTES)
        if not positions_given and not native:
            positions = torch.cat([torch.arange(p0, p0 + n, device=x.device) for _, n, p0 in segs])
            positions = positions.unsqueeze(0).expand(B, -1)
        fused = None
        if not native and train is None and dt == torch.bfloat16 and self.fused_gemm:
            # the projections and their epilogue in one tensor-core GEMM (no projection tensor)
            Wp, bp = self.fused_projection_tiles()
            fused = ops.proj_fused(dims, Wp, bp, x.reshape(B * L, self.d_model), B, L, positions,
                                   self.rotary_emb.cos_cached, self.rotary_emb.sin_cached,
                                   kv_out=store.kv[:, past_len:past_len + L] if store is not None else None,
                                   ki_out=store.ki[:, past_len:past_len + L] if store is not None else None)
        if fused is None:
            # the stacked weights are built (and kept) only for the paths that use them, so a layer on
            # the fused GEMM holds one copy of its weights in the GEMM's row order, not two
            W, bvec, layout = self.fused_projection()
            proj = torch.addmm(bvec, x.reshape(B * L, self.d_model), W.t())
        if not self.training:
            # the gates' analysis output (last_gate_scores), computed from their logits when read
            if fused is None:
                if self.value_gate is not None:
                    self.value_gate._set_pending_logits(proj[:, layout.g2:layout.g2 + Hk * D].view(B, L, Hk, D))
                if self.output_gate is not None:
                    self.output_gate._set_pending_logits(proj[:, layout.g1:layout.g1 + H * D].view(B, L, H, D))
            else:
                for gate, shape in ((self.value_gate, (B, L, Hk, D)), (self.output_gate, (B, L, H, D))):
                    if gate is not None:
                        gate._set_pending_logits(_LazyLogits(x, gate.gate_proj.weight, gate.gate_proj.bias, shape))
        if native:
            # everything between the two GEMMs in one native call, scratch kept on the store
            dims, tp, idx_bias = self._step_constants()
            nbytes = ops.decode_workspace_bytes(dims, tp, dt, B, L, store.capacity)
            attn = ops.decode_attend(dims, layout, tp, proj, B, L, past_len, positions if positions_given else None,
                                     self.rotary_emb.cos_cached, self.rotary_emb.sin_cached, store.kv, store.ki,
                                     idx_bias, self.indexer.scale, self.scale, store.scratch((B, L), nbytes),
                                     allreduce=(self.sequence_shards.allreduce if self.sequence_shards is not None
                                                and cfg.use_adaptive_k else None))
            out = F.linear(attn.view(B, L, H * D), self.o_proj.weight)
            present = None
            if use_cache:
                store.filled = n_all
                present = store.view(n_all)
            return out, present, None
        mark("proj_gemm")
        if fused is not None:
            q, kv, g1, w, shift, qI, kI = fused
            proj = None
        else:
            q, kv, g1, w, shift = ops.proj_epilogue(
                dims, layout, proj, positions, self.rotary_emb.cos_cached, self.rotary_emb.sin_cached,
                self.output_gate is not None, return_kv=True,
                kv_out=store.kv[:, past_len:past_len + L] if store is not None else None,
                ki_out=store.ki[:, past_len:past_len + L] if store is not None else None)
            proj3 = proj.view(B, L, proj.shape[1])
            qI = proj3[..., layout.qi:layout.qi + HI * dI]
            kI = proj3[..., layout.ki:layout.ki + dI]
        mark("proj_epilogue")
        q = q.view(B, L, H, D)
        kv = kv.view(B, L, 2, Hk, D)  # k and v interleaved per token

        indexer_keys = None
        kv_finish = None
        present = None
        if store is not None:
            # K, V and k^I of every cached and new token, in place in the store
            n = past_len + L
            kv_all, kI_all, q_pos0 = store.kv[:, :n], store.ki[:, :n], past_len
            indexer_keys = kI_all
            if use_cache:
                store.filled = n
                present = store.view(n)
        elif sp is not None:
            # every rank needs all keys up to its last query, in sequence order: k^I now (the
            # indexer reads it), K/V asynchronously (only the SDPA reads them), so that their
            # transfer overlaps the indexer
            kI_all = sp.gather(kI)
            kv_finish = sp.gather_async(kv)
            kv_all = None
            q_pos0 = segs[0][2]
            indexer_keys = kI_all
        elif past_key_value is None:
            # no cache kept
            kv_all, kI_all, q_pos0 = kv, kI, 0
        else:
            # a plain (k, v) cache (no indexer keys): the reference concatenates it and scores
            # the new tokens only (gated_sparse_attention.py:188-213), selecting among
            # positions [0, L)
            past_kv = torch.stack([past_key_value[0], past_key_value[1]], dim=2)
            kv_all = torch.cat([past_kv, kv], dim=1)
            kI_all, q_pos0 = kI, 0
        if kv_finish is None:
            k_all, v_all = kv_all[:, :, 0], kv_all[:, :, 1]
            if use_cache and present is None:
                present = GSAKVCache(k_all, v_all, indexer_keys, kv_all)
        mark("kv")

        n_cols = kI_all.shape[1]
        k_eff = min(cfg.k_max, n_cols) if cfg.use_adaptive_k else min(cfg.k_base, n_cols)
        # the candidates of a row: its k_eff best keys (exact) or its threshold survivors, a
        # superset in the same ascending order; the final selection takes k_t from either
        survivors = (self.selection_path == "auto" and not output_attentions
                     and ops.survivors_eligible(dims, k_eff, True))
        select_fn = ops.indexer_survivors if survivors else ops.indexer_select
        cand_ld = ops.SURVIVOR_CAP if survivors else k_eff
        n_chunks = 0  # indexer launches (query chunks) of this forward, for the launch count
        if len(segs) == 1:
            cand_idx, cand_score, cand_count, stats = select_fn(
                dims, qI, kI_all, w, self.indexer.bias, self.indexer.scale, shift, k_eff,
                q_pos0=q_pos0, causal=True)
            n_chunks = ops.last_chunk_count
        else:
            # one indexer pass per query segment, each with its own causal offset
            R = B * L
            cand_idx = torch.zeros(R, cand_ld, device=x.device, dtype=torch.int32)
            cand_score = torch.empty(R, cand_ld, device=x.device, dtype=torch.float32)
            cand_count = torch.empty(R, device=x.device, dtype=torch.int32)
            stats = torch.zeros(R, 3, device=x.device, dtype=torch.float64)
            wv = w.view(L, HI)
            for l0, n, p0 in segs:
                select_fn(dims, qI[:, l0:l0 + n], kI_all, wv[l0:l0 + n], self.indexer.bias,
                          self.indexer.scale, shift[l0:l0 + n], k_eff, q_pos0=p0, causal=True,
                          row_stats=stats[l0:l0 + n],
                          out=(cand_idx[l0:l0 + n], cand_score[l0:l0 + n], cand_count[l0:l0 + n]))
                n_chunks += ops.last_chunk_count
        mark("indexer_topk")
        if cfg.use_adaptive_k:
            var, total = ops.row_variance(stats, n_cols, dt, shift)
            if sp is not None:
                total = sp.allreduce(total)
            elif self.sequence_shards is not None:
                total = self.sequence_shards.allreduce(total)
        else:
            var = total = None
        kt = ops.adaptive_k(stats, var, total, n_cols, dt, cfg.k_base, cfg.k_min, cfg.k_max,
                            cfg.use_adaptive_k, cfg.adaptive_k_temperature)
        sel, cnt, mask = ops.select_finalize(cand_idx, cand_score, cand_count, kt, want_mask=output_attentions,
                                             sel_ld=k_eff)
        mark("adaptive_k_select")
        if kv_finish is not None:
            kv_all = kv_finish()
            mark("kv_gather_wait")
            k_all, v_all = kv_all[:, :, 0], kv_all[:, :, 1]
            present = GSAKVCache(k_all, v_all, indexer_keys, kv_all) if use_cache else None
        lse = None
        if train is None and output_attentions:
            # the gated output and each (row, head)'s log-sum-exp, from which the probabilities follow
            attn, lse = ops.sparse_sdpa_lse_gated(dims, q, k_all, v_all, sel, cnt, g1, self.scale)
        elif train is None:
            attn = ops.sparse_sdpa(dims, q, k_all, v_all, sel, cnt, g1, self.scale)
        else:
            # ungated output and softmax statistics kept for the backward; the gate applied as the
            # fused epilogue applies it (one product rounded to the dtype)
            O, lse = ops.sparse_sdpa_lse(dims, q, k_all, v_all, sel, cnt, self.scale)
            attn = O * g1.view_as(O) if g1 is not None else O
            train.update(dims=dims, layout=layout, proj=proj, positions=positions, q=q, k=k_all, v=v_all,
                         sel=sel, cnt=cnt, O=O, lse=lse, g1=g1, gated=attn)
        mark("sparse_sdpa")
        out = F.linear(attn.view(B, L, H * D), self.o_proj.weight)
        mark("o_proj")
        if capture is not None:
            # the indexer's inputs and its query segments (local start, rows, first position)
            capture.update(qI=qI, kI=kI_all, w=w, shift=shift, bias=self.indexer.bias,
                           idx_scale=self.indexer.scale,
                           idx_segments=list(segs) if len(segs) > 1 else [(0, L, q_pos0)])
            capture.update(dims=dims, q=q, k=k_all, v=v_all, sel=sel, cnt=cnt, gate=g1, k_t=kt, attn=attn,
                           var=var, var_total=total,
                           n_chunks=n_chunks, candidate_path="survivors" if survivors else "exact",
                           survivor_pass=ops.last_survivor_path if survivors else None)

        weights = None
        if output_attentions:
            weights = self._attention_weights(dims, q, k_all, cand_idx, cand_score, cand_count, mask, lse)
        return out, present, weights

    def _attention_weights(self, dims, q, k, cand_idx, cand_score, cand_count, mask, lse):
        """Softmax weights [B, L, H, k_eff] (analysis output; gated_sparse_attention.py:268-285).

        Like the reference's, position p of a row holds the weight of its p-th best candidate
        (scores descending, adaptive_topk.py:177; ties lower column first) and the kept keys come
        first; positions past k_t are 0.  The probabilities come from a kernel pass over the kept
        keys with the SDPA's own log-sum-exp."""
        B, L, H, D = q.shape
        R, k_eff = cand_idx.shape
        if R > 65535 or R * H * k_eff > (1 << 31):
            raise NotImplementedError("output_attentions is limited to small shapes")
        pos = torch.arange(k_eff, device=q.device).view(1, -1)
        valid = pos < cand_count.view(-1, 1).long()
        key = cand_score.masked_fill(~valid, float("-inf"))
        order = torch.sort(key, dim=1, descending=True, stable=True).indices
        idx = torch.gather(cand_idx, 1, order).masked_fill(~torch.gather(valid, 1, order), 0)
        keep = torch.gather(mask, 1, order) & torch.gather(valid, 1, order).to(mask.dtype)
        return ops.sparse_sdpa_probs(dims, q, k, idx, keep, lse, self.scale)
