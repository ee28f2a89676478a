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


class GSALlamaModel(nn.Module):
    """Token embedding, decoder layers and the final norm (gsa_llama.py:134-242)."""

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

    def forward(self, input_ids: torch.Tensor, positions: Optional[torch.Tensor] = None,
                attention_mask: Optional[torch.Tensor] = None,
                past_key_values: Optional[Tuple[Tuple[torch.Tensor, torch.Tensor], ...]] = None,
                use_cache: bool = False, output_attentions: bool = False,
                output_hidden_states: bool = False) -> GSAModelOutput:
        batch_size, seq_len = input_ids.shape
        hidden_states = self.embed_tokens(input_ids)
        if positions is None:
            past_len = past_key_values[0][0].shape[1] if past_key_values else 0
            positions = torch.arange(past_len, past_len + seq_len,
                                     device=input_ids.device).unsqueeze(0).expand(batch_size, -1)
        all_hidden_states = () if output_hidden_states else None
        all_attentions = () if output_attentions else None
        next_cache = () if use_cache else None
        for i, layer in enumerate(self.layers):
            if output_hidden_states:
                all_hidden_states = all_hidden_states + (hidden_states,)
            past_key_value = past_key_values[i] if past_key_values else None
            if self.gradient_checkpointing and self.training:
                hidden_states, present_key_value, attn_weights = torch.utils.checkpoint.checkpoint(
                    layer, hidden_states, positions, attention_mask, past_key_value, use_cache, output_attentions,
                    use_reentrant=False)
            else:
                hidden_states, present_key_value, attn_weights = layer(
                    hidden_states, positions=positions, attention_mask=attention_mask,
                    past_key_value=past_key_value, use_cache=use_cache, output_attentions=output_attentions)
            if use_cache:
                next_cache = next_cache + (present_key_value,)
            if output_attentions:
                all_attentions = all_attentions + (attn_weights,)
        hidden_states = self.norm(hidden_states)
        if output_hidden_states:
            all_hidden_states = all_hidden_states + (hidden_states,)
        return GSAModelOutput(last_hidden_state=hidden_states, past_key_values=next_cache,
                              hidden_states=all_hidden_states, attentions=all_attentions)


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
        outputs = self.model(input_ids=input_ids, positions=positions, attention_mask=attention_mask,
                             past_key_values=past_key_values, use_cache=use_cache,
                             output_attentions=output_attentions, output_hidden_states=output_hidden_states)
        logits = self.lm_head(outputs.last_hidden_state)
        loss = None
        if labels is not None:
            shift_logits = logits[..., :-1, :].contiguous()
            shift_labels = labels[..., 1:].contiguous()
            loss = F.cross_entropy(shift_logits.view(-1, self.config.vocab_size), shift_labels.view(-1),
                                   ignore_index=-100)
        return GSACausalLMOutput(loss=loss, logits=logits, past_key_values=outputs.past_key_values,
                                 hidden_states=outputs.hidden_states, attentions=outputs.attentions)

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 100, temperature: float = 1.0,
                 top_p: float = 0.9, top_k: int = 50, do_sample: bool = True, pad_token_id: Optional[int] = None,
                 eos_token_id: Optional[int] = None) -> torch.Tensor:
        """Autoregressive sampling (gsa_llama.py:332-430).  Each step after the first feeds the
        last token against the layers' KV caches, which carry the indexer keys and grow in place."""
        past_key_values = None
        generated = input_ids
        for _ in range(max_new_tokens):
            curr_input = generated[:, -1:] if past_key_values is not None else generated
            outputs = self.forward(input_ids=curr_input, past_key_values=past_key_values, use_cache=True)
            past_key_values = outputs.past_key_values
            logits = outputs.logits[:, -1, :]
            if temperature != 1.0:
                logits = logits / temperature
            if top_k > 0:
                indices_to_remove = logits < torch.topk(logits, top_k)[0][..., -1, None]
                logits[indices_to_remove] = float("-inf")
            if top_p < 1.0:
                sorted_logits, sorted_indices = torch.sort(logits, descending=True)
                cumulative_probs = torch.cumsum(F.softmax(sorted_logits, dim=-1), dim=-1)
                sorted_indices_to_remove = cumulative_probs > top_p
                sorted_indices_to_remove[..., 1:] = sorted_indices_to_remove[..., :-1].clone()
                sorted_indices_to_remove[..., 0] = 0
                indices_to_remove = sorted_indices_to_remove.scatter(1, sorted_indices, sorted_indices_to_remove)
                logits[indices_to_remove] = float("-inf")
            if do_sample:
                next_token = torch.multinomial(F.softmax(logits, dim=-1), num_samples=1)
            else:
                next_token = torch.argmax(logits, dim=-1, keepdim=True)
            generated = torch.cat([generated, next_token], dim=-1)
            if eos_token_id is not None and (next_token == eos_token_id).all():
                break
        return generated

    @classmethod
    def from_pretrained(cls, path: str) -> "GSALlamaForCausalLM":
        """config.json + model.safetensors (or pytorch_model.bin), as the reference saves them."""
        import json
        from pathlib import Path

        path = Path(path)
        with open(path / "config.json", "r") as f:
            config = GSAConfig.from_dict(json.load(f))
        model = cls(config)
        if (path / "model.safetensors").exists():
            from safetensors.torch import load_file
            state_dict = load_file(path / "model.safetensors")
        else:
            state_dict = torch.load(path / "pytorch_model.bin", map_location="cpu")
        model.load_state_dict(state_dict)
        return model

    def save_pretrained(self, path: str):
        from pathlib import Path

        from safetensors.torch import save_file

        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        self.config.save_pretrained(path)
        save_file(self.state_dict(), path / "model.safetensors")


GSAForCausalLM = GSALlamaForCausalLM
