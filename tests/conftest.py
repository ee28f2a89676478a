import json
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "gated-sparse-attention_b200", ROOT / "oracle", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str):
    """(tensors dict, metadata dict with parsed config) of a golden fixture."""
    from safetensors import safe_open

    with safe_open(str(GOLDEN / f"{name}.safetensors"), "pt") as f:
        meta = dict(f.metadata())
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    meta["config"] = json.loads(meta["config"])
    meta["param_checksums"] = json.loads(meta["param_checksums"])
    return tensors, meta


def golden_inputs(meta):
    """Rebuild the fixture's module weights (seeded init) and input x."""
    from gsa_b200 import GSAConfig, GatedSparseAttention

    cfg = GSAConfig(**meta["config"])
    dtype = getattr(torch, meta["dtype"])
    torch.manual_seed(int(meta["weight_seed"]))
    m = GatedSparseAttention(cfg).eval().to(dtype)
    gen = torch.Generator().manual_seed(int(meta["input_seed"]))
    B, L = int(meta["batch"]), int(meta["seq_len"])
    x = torch.randn(B, L, cfg.d_model, generator=gen).to(dtype)
    return cfg, m, x


GOLDEN_NAMES = ["tiny_fp32_b2_l192", "tiny_bf16_b2_l192", "tiny_fixedk_nogate_fp32_l128",
                "c1_fp32_l2048", "w4096_bf16_l384"]


@pytest.fixture(scope="session")
def cuda_ok():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True
