"""gsa_b200: the Gated Sparse Attention forward path on NVIDIA B200 (sm_100a).

Drop-in for the reference package's attention API (``from gsa import GSAConfig,
GatedSparseAttention``): same classes, arguments, parameter names and outputs, computed by the
hand-written CUDA kernels of ``libgsa_b200.so`` through its C ABI (include/gsa_b200.h).
"""

from .config import GSAConfig
from .attention import (
    AdaptiveTopKSelector,
    GatedLightningIndexer,
    GatedSparseAttention,
    GSAKVCache,
    OutputGate,
    RotaryEmbedding,
    ValueGate,
    apply_rotary_pos_emb,
)

from .models import (
    GSACausalLMOutput,
    GSADecoderLayer,
    GSAForCausalLM,
    GSALlamaForCausalLM,
    GSALlamaModel,
    GSAMlp,
    GSAModelOutput,
    RMSNorm,
)

__version__ = "0.1.0"
__all__ = [
    "GSAConfig",
    "GatedSparseAttention",
    "GatedLightningIndexer",
    "AdaptiveTopKSelector",
    "ValueGate",
    "OutputGate",
    "RotaryEmbedding",
    "apply_rotary_pos_emb",
    "GSAKVCache",
    "RMSNorm",
    "GSAMlp",
    "GSADecoderLayer",
    "GSAModelOutput",
    "GSACausalLMOutput",
    "GSALlamaModel",
    "GSALlamaForCausalLM",
    "GSAForCausalLM",
]
