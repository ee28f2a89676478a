"""The reference's LLaMA-style model around the attention, on the B200 kernels.

Class names, constructor arguments, submodule and parameter names, return types and outputs follow
``gsa/models/gsa_llama.py`` (alfredcs/Gated-Sparse-Attention):

  RMSNorm               gsa_llama.py:18-30
  GSAMlp                gsa_llama.py:33-46   (SwiGLU)
  GSADecoderLayer       gsa_llama.py:49-112
  GSAModelOutput        gsa_llama.py:115-121
  GSACausalLMOutput     gsa_llama.py:124-131
  GSALlamaModel         gsa_llama.py:134-242
  GSALlamaForCausalLM   gsa_llama.py:245-469 (forward, generate, from_pretrained, save_pretrained)

Submodules are created and initialised in the reference's order, so ``torch.manual_seed(s)``
before construction gives the reference's weights and state dicts load either way.

Without autograd the decoder layer runs: the fused residual-add + RMSNorm kernel, the attention
layer (its own kernels), and a SwiGLU MLP of one GEMM over the concatenated gate/up weights, the
silu-product kernel and the down GEMM (cuBLAS).  Under autograd the norm and MLP use the
reference's torch formulas (differentiable) around the attention's autograd function.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .attention import GatedSparseAttention
from .config import GSAConfig


def _fused(x: torch.Tensor, *params) -> bool:
    """Whether the kernels run (CUDA tensors, no gradient wanted)."""
    if not x.is_cuda:
        raise RuntimeError("the B200 GSA modules run on CUDA tensors only")
    return not (torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in params)))


class RMSNorm(nn.Module):
    """Root mean square layer normalisation (gsa_llama.py:18-30)."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def _norm(self, x: torch.Tensor) -> torch.Tensor:
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _fused(x, self.weight):
            return ops.add_rmsnorm(x, None, self.weight, self.eps, want_sum=False)[1]
        return self._norm(x.float()).type_as(x) * self.weight

    def add_forward(self, residual: torch.Tensor, a: torch.Tensor):
        """(residual + a, RMSNorm(residual + a)) in one pass over the row."""
        if _fused(residual, self.weight) and not a.requires_grad:
            return ops.add_rmsnorm(residual, a, self.weight, self.eps)
        h = residual + a
        return h, self(h)


class GSAMlp(nn.Module):
    """SwiGLU MLP (gsa_llama.py:33-46): down(silu(gate(x)) * up(x))."""

    def __init__(self, config: GSAConfig):
        super().__init__()
        self.d_model = config.d_model
        self.d_ffn = config.d_ffn
        self.gate_proj = nn.Linear(self.d_model, self.d_ffn, bias=False)
        self.up_proj = nn.Linear(self.d_model, self.d_ffn, bias=False)
        self.down_proj = nn.Linear(self.d_ffn, self.d_model, bias=False)
        self._gu = None

    def _gate_up(self) -> torch.Tensor:
        """[W_gate; W_up] for one GEMM, rebuilt when either weight changes."""
        g, u = self.gate_proj.weight, self.up_proj.weight
        key = (g.data_ptr(), g._version, u.data_ptr(), u._version)
        if self._gu is None or self._gu[0] != key:
            self._gu = (key, torch.cat([g.detach(), u.detach()], 0).contiguous())
        return self._gu[1]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _fused(x, self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight):
            gu = F.linear(x, self._gate_up())
            return F.linear(ops.silu_mul(gu), self.down_proj.weight)
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class GSADecoderLayer(nn.Module):
    """Pre-norm decoder layer: x + GSA(RMSNorm(x)), then h + MLP(RMSNorm(h)) (gsa_llama.py:49-112)."""

    def __init__(self, config: GSAConfig, layer_idx: int):
        super().__init__()
        self.layer_idx = layer_idx
        self.input_layernorm = RMSNorm(config.d_model, eps=config.norm_eps)
        self.self_attn = GatedSparseAttention(config)
        self.post_attention_layernorm = RMSNorm(config.d_model, eps=config.norm_eps)
        self.mlp = GSAMlp(config)

    def forward(self, hidden_states: torch.Tensor, positions: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                past_key_value: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                use_cache: bool = False, output_attentions: bool = False):
        residual = hidden_states
        hidden_states = self.input_layernorm(hidden_states)
        attn_output, present_key_value, attn_weights = self.self_attn(
            hidden_states, positions=positions, attention_mask=attention_mask, past_key_value=past_key_value,
            use_cache=use_cache, output_attentions=output_attentions)
        hidden_states, normed = self.post_attention_layernorm.add_forward(residual, attn_output)
        mlp_out = self.mlp(normed)
        if _fused(hidden_states, *self.parameters()) and not mlp_out.requires_grad:
            hidden_states = ops.add_rmsnorm(hidden_states, mlp_out, None, 0.0, want_norm=False)[0]
        else:
            hidden_states = hidden_states + mlp_out
        return hidden_states, present_key_value, attn_weights


@dataclass
class GSAModelOutput:
    """Output of GSALlamaModel (gsa_llama.py:115-121)."""
    last_hidden_state: torch.Tensor
    past_key_values: Optional[Tuple[Tuple[torch.Tensor, torch.Tensor], ...]] = None
    hidden_states: Optional[Tuple[torch.Tensor, ...]] = None
    attentions: Optional[Tuple[torch.Tensor, ...]] = None


@dataclass
class GSACausalLMOutput:
    """Output of GSALlamaForCausalLM (gsa_llama.py:124-131)."""
    loss: Optional[torch.Tensor] = None
    logits: torch.Tensor = None
    past_key_values: Optional[Tuple[Tuple[torch.Tensor, torch.Tensor], ...]] = None
    hidden_states: Optional[Tuple[torch.Tensor, ...]] = None
    attentions: Optional[Tuple[torch.Tensor, ...]] = None


def _cache_length(past_key_values) -> int:
    """Tokens already held by the first layer's cache (0 without caches)."""
    if not past_key_values or past_key_values[0] is None:
        return 0
    return past_key_values[0][0].shape[1]


class GSALlamaModel(nn.Module):
    """Token embedding, decoder layers and the final norm (gsa_llama.py:134-242).

    The layers' caches are the attention layers' in-place stores: a cache returned by one call is a
    view of a buffer with headroom, and passing it back lets the next call append K, V and the
    indexer keys in place (``allocate_caches`` sizes them up front)."""

    def __init__(self, config: GSAConfig):
        super().__init__()
        self.config = config
        self.vocab_size = config.vocab_size
        self.n_layers = config.n_layers
        self.embed_tokens = nn.Embedding(config.vocab_size, config.d_model)
        self.layers = nn.ModuleList([GSADecoderLayer(config, layer_idx=i) for i in range(config.n_layers)])
        self.norm = RMSNorm(config.d_model, eps=config.norm_eps)
        self.gradient_checkpointing = False
        self._init_weights()

    def _init_weights(self):
        nn.init.normal_(self.embed_tokens.weight, std=self.config.initializer_range)

    def allocate_caches(self, batch_size: int, capacity: int):
        """Empty per-layer caches with room for ``capacity`` tokens of each sequence; pass them as
        ``past_key_values`` (with ``use_cache=True``) and every call writes into them in place."""
        return tuple(layer.self_attn.allocate_cache(batch_size, capacity) for layer in self.layers)

    def _layer_call(self, layer, h, positions, attention_mask, cache, use_cache, output_attentions):
        if self.gradient_checkpointing and self.training:
            return torch.utils.checkpoint.checkpoint(layer, h, positions, attention_mask, cache, use_cache,
                                                     output_attentions, use_reentrant=False)
        return layer(h, positions=positions, attention_mask=attention_mask, past_key_value=cache,
                     use_cache=use_cache, output_attentions=output_attentions)

    def forward(self, input_ids: torch.Tensor, positions: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                past_key_values: Optional[Tuple[Tuple[torch.Tensor, torch.Tensor], ...]] = None,
                use_cache: bool = False, output_attentions: bool = False,
                output_hidden_states: bool = False) -> GSAModelOutput:
        B, L = input_ids.shape
        if positions is None:
            start = _cache_length(past_key_values)
            positions = (torch.arange(L, device=input_ids.device) + start).expand(B, L)
        caches = list(past_key_values) if past_key_values else [None] * len(self.layers)
        h = self.embed_tokens(input_ids)
        seen, presents, weights = [], [], []
        for layer, cache in zip(self.layers, caches):
            seen.append(h)
            h, present, attn = self._layer_call(layer, h, positions, attention_mask, cache, use_cache,
                                                output_attentions)
            presents.append(present)
            weights.append(attn)
        h = self.norm(h)
        seen.append(h)
        return GSAModelOutput(last_hidden_state=h,
                              past_key_values=tuple(presents) if use_cache else None,
                              hidden_states=tuple(seen) if output_hidden_states else None,
                              attentions=tuple(weights) if output_attentions else None)


def next_token_loss(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    """Mean cross-entropy of token t+1 predicted at position t; labels of -100 do not count
    (gsa_llama.py:323-336)."""
    V = logits.shape[-1]
    return F.cross_entropy(logits[:, :-1].reshape(-1, V), labels[:, 1:].reshape(-1), ignore_index=-100)


def filter_logits(logits: torch.Tensor, temperature: float = 1.0, top_k: int = 0,
                  top_p: float = 1.0) -> torch.Tensor:
    """The sampling filter of generate (gsa_llama.py:388-410) as one function, on a copy of [B, V]
    logits: divide by the temperature; keep the logits not below the k-th largest (ties at it kept);
    then nucleus filtering -- in descending order (torch.sort), a token is dropped when the
    probabilities of the tokens ahead of it already sum to more than top_p (so the most likely
    token always stays).  Dropped logits become -inf."""
    out = logits / temperature if temperature != 1.0 else logits.clone()
    if top_k > 0:
        kth = torch.topk(out, top_k, dim=-1).values[..., -1:]
        out = out.masked_fill(out < kth, float("-inf"))
    if top_p < 1.0:
        srt, order = torch.sort(out, dim=-1, descending=True)
        ahead = torch.cumsum(F.softmax(srt, dim=-1), dim=-1)
        # probability mass strictly ahead of each sorted position (the inclusive sum, shifted by one)
        ahead = torch.cat([torch.zeros_like(ahead[..., :1]), ahead[..., :-1]], dim=-1)
        keep = torch.zeros_like(out, dtype=torch.bool).scatter(-1, order, ahead <= top_p)
        out = out.masked_fill(~keep, float("-inf"))
    return out


def sample_tokens(logits: torch.Tensor, do_sample: bool) -> torch.Tensor:
    """[B, 1] next tokens: a draw from softmax(logits) (torch.multinomial on the global generator), or
    the argmax."""
    if do_sample:
        return torch.multinomial(F.softmax(logits, dim=-1), num_samples=1)
    return torch.argmax(logits, dim=-1, keepdim=True)


def decode_loop(step, input_ids: torch.Tensor, max_new_tokens: int, temperature: float, top_k: int,
                top_p: float, do_sample: bool, eos_token_id: Optional[int]) -> torch.Tensor:
    """The token loop of generate: ``step(tokens, first)`` returns the [B, V] logits of the last
    position after feeding ``tokens`` (the whole prompt when ``first``, else the newest token)."""
    tokens = [input_ids]
    feed, first = input_ids, True
    for _ in range(max_new_tokens):
        logits = filter_logits(step(feed, first), temperature, top_k, top_p)
        nxt = sample_tokens(logits, do_sample)
        tokens.append(nxt)
        feed, first = nxt, False
        if eos_token_id is not None and bool((nxt == eos_token_id).all()):
            break
    return torch.cat(tokens, dim=-1)


class GSALlamaForCausalLM(nn.Module):
    """GSALlamaModel with the LM head, next-token loss and sampling (gsa_llama.py:245-469)."""

    def __init__(self, config: GSAConfig):
        super().__init__()
        self.config = config
        self.model = GSALlamaModel(config)
        self.lm_head = nn.Linear(config.d_model, config.vocab_size, bias=False)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight
        self._init_weights()

    def _init_weights(self):
        if not self.config.tie_word_embeddings:
            nn.init.normal_(self.lm_head.weight, std=self.config.initializer_range)

    def forward(self, input_ids: torch.Tensor, positions: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None, labels: Optional[torch.Tensor] = None,
                past_key_values: Optional[Tuple[Tuple[torch.Tensor, torch.Tensor], ...]] = None,
                use_cache: bool = False, output_attentions: bool = False,
                output_hidden_states: bool = False) -> GSACausalLMOutput:
        base = self.model(input_ids=input_ids, positions=positions, attention_mask=attention_mask,
                          past_key_values=past_key_values, use_cache=use_cache,
                          output_attentions=output_attentions, output_hidden_states=output_hidden_states)
        logits = self.lm_head(base.last_hidden_state)
        return GSACausalLMOutput(loss=None if labels is None else next_token_loss(logits, labels), logits=logits,
                                 past_key_values=base.past_key_values, hidden_states=base.hidden_states,
                                 attentions=base.attentions)

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 100, temperature: float = 1.0,
                 top_p: float = 0.9, top_k: int = 50, do_sample: bool = True, pad_token_id: Optional[int] = None,
                 eos_token_id: Optional[int] = None) -> torch.Tensor:
        """Autoregressive decoding (gsa_llama.py:344-430), same arguments and sampling.  Every layer's
        cache is allocated once for the prompt plus ``max_new_tokens``; the prompt and then each new
        token are written into it in place, and each step scores the new token against every cached
        indexer key."""
        caches = [self.model.allocate_caches(input_ids.shape[0], input_ids.shape[1] + max_new_tokens)]

        def step(tokens, first):
            out = self.forward(input_ids=tokens, past_key_values=caches[0], use_cache=True)
            caches[0] = out.past_key_values
            return out.logits[:, -1, :]

        return decode_loop(step, input_ids, max_new_tokens, temperature, top_k, top_p, do_sample, eos_token_id)

    _WEIGHT_FILES = ("model.safetensors", "pytorch_model.bin")

    @classmethod
    def from_pretrained(cls, path: str) -> "GSALlamaForCausalLM":
        """A model directory written by save_pretrained (or the reference's): config.json and
        model.safetensors, else pytorch_model.bin (gsa_llama.py:432-458)."""
        from pathlib import Path

        root = Path(path)
        model = cls(GSAConfig.from_pretrained(str(root)))
        found = [root / n for n in cls._WEIGHT_FILES if (root / n).exists()]
        if not found:
            raise FileNotFoundError(f"no {' or '.join(cls._WEIGHT_FILES)} in {root}")
        if found[0].suffix == ".safetensors":
            from safetensors.torch import load_file
            state = load_file(str(found[0]))
        else:
            state = torch.load(found[0], map_location="cpu")
        model.load_state_dict(state)
        return model

    def save_pretrained(self, path: str):
        """config.json and model.safetensors into ``path`` (gsa_llama.py:460-469)."""
        from safetensors.torch import save_file

        self.config.save_pretrained(path)
        save_file(self.state_dict(), f"{path}/model.safetensors")


GSAForCausalLM = GSALlamaForCausalLM
