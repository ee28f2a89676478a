"""GSAConfig: the hyper-parameters of one GSA layer.

Same field names, defaults and validation as the reference's ``GSAConfig``
(gsa/config.py:9-134), so that configs, ``from_dict`` payloads and ``config.json`` files move
between the two unchanged.  ``GSATrainingConfig`` (gsa/config.py:137-177) belongs to the
training loop and is not part of this package.
"""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, Optional


@dataclass
class GSAConfig:
    # layer widths (gsa/config.py:24-27); d_head defaults to d_model // n_heads
    d_model: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    d_head: Optional[int] = None

    # model-level fields carried for compatibility (gsa/config.py:30-32)
    n_layers: int = 32
    d_ffn: int = 11008
    vocab_size: int = 128256

    # indexer (gsa/config.py:35-37)
    d_indexer: int = 64
    n_indexer_heads: int = 4
    indexer_activation: str = "sigmoid"

    # sparsity (gsa/config.py:40-44)
    k_base: int = 2048
    k_min: int = 256
    k_max: int = 4096
    use_adaptive_k: bool = True
    adaptive_k_temperature: float = 1.0

    # gates (gsa/config.py:47-50)
    use_value_gate: bool = True
    use_output_gate: bool = True
    gate_activation: str = "sigmoid"
    gate_bias_init: float = 0.5

    # RoPE (gsa/config.py:53-55)
    rope_base: float = 10000.0
    rope_scaling: Optional[Dict[str, Any]] = None
    max_position_embeddings: int = 131072

    # training-time knobs kept for config compatibility (gsa/config.py:58-66)
    dense_residual_alpha: float = 0.0
    use_indexer_warmup: bool = True
    indexer_warmup_steps: int = 1000
    use_flash_attention: bool = True
    use_triton_kernels: bool = True
    attention_dropout: float = 0.0
    hidden_dropout: float = 0.0

    # model-level (gsa/config.py:69-74)
    norm_eps: float = 1e-5
    use_rms_norm: bool = True
    tie_word_embeddings: bool = False
    initializer_range: float = 0.02

    def __post_init__(self):
        # the same checks, in the same order and with the same AssertionError, as
        # gsa/config.py:76-95
        if self.d_head is None:
            self.d_head = self.d_model // self.n_heads
        assert self.d_model % self.n_heads == 0, (
            f"d_model ({self.d_model}) must be divisible by n_heads ({self.n_heads})")
        assert self.n_heads % self.n_kv_heads == 0, (
            f"n_heads ({self.n_heads}) must be divisible by n_kv_heads ({self.n_kv_heads})")
        assert self.k_min <= self.k_base <= self.k_max, (
            f"k_min ({self.k_min}) <= k_base ({self.k_base}) <= k_max ({self.k_max}) required")
        assert self.indexer_activation in ["sigmoid", "relu"], (
            f"indexer_activation must be 'sigmoid' or 'relu', got {self.indexer_activation}")
        assert self.gate_activation in ["sigmoid", "tanh", "silu"], (
            f"gate_activation must be 'sigmoid', 'tanh', or 'silu', got {self.gate_activation}")

    @classmethod
    def from_dict(cls, config_dict: Dict[str, Any]) -> "GSAConfig":
        """Build from a dict, ignoring unknown keys."""
        return cls(**{k: v for k, v in config_dict.items() if k in cls.__dataclass_fields__})

    def to_dict(self) -> Dict[str, Any]:
        return {k: getattr(self, k) for k in self.__dataclass_fields__}

    @classmethod
    def from_pretrained(cls, model_name_or_path: str) -> "GSAConfig":
        """Load ``config.json`` from a local directory (no hub access in this package)."""
        path = Path(model_name_or_path) / "config.json"
        if not path.exists():
            raise FileNotFoundError(f"{path} not found")
        with open(path) as f:
            return cls.from_dict(json.load(f))

    def save_pretrained(self, save_directory: str) -> None:
        out = Path(save_directory)
        out.mkdir(parents=True, exist_ok=True)
        with open(out / "config.json", "w") as f:
            json.dump(self.to_dict(), f, indent=2)
