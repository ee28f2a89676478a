"""The bf16 projection epilogue has a 16-byte vector kernel and a scalar one (any alignment).
Both evaluate the same ops with the same roundings, so their outputs must agree bit for bit:
the vector kernel runs on an aligned projection buffer, the scalar kernel on a copy of it shifted
by one element.  Covered: bf16 and fp32 RoPE tables, sigmoid / tanh / silu gates, G1 on and off."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("tab_dtype,gate_act,has_g1", [
    (torch.bfloat16, "sigmoid", True),
    (torch.float32, "tanh", True),
    (torch.bfloat16, "silu", False),
])
def test_vector_and_scalar_epilogue_agree(cuda_ok, tab_dtype, gate_act, has_g1):
    from gsa_b200 import ops
    from gsa_b200._lib import ProjLayout

    H, Hk, D, HI, T = 8, 2, 128, 8, 333
    dims = ops.make_dims(1024, H, Hk, D, HI, 64, gate_act=gate_act)
    # column layout of one fused projection row: q | k | v | g2 | g1 | qI | kI | w
    off, cols = {}, 0
    for name, width in (("q", H * D), ("k", Hk * D), ("v", Hk * D), ("g2", Hk * D), ("g1", H * D),
                        ("qi", HI * 64), ("ki", 64), ("wi", HI)):
        off[name] = cols
        cols += width
    layout = ProjLayout(off["q"], off["k"], off["v"], off["g2"], off["g1"] if has_g1 else -1, off["qi"],
                        off["ki"], off["wi"])
    ncat = (cols + 63) // 64 * 64
    g = torch.Generator().manual_seed(3)
    proj = (torch.randn(T, ncat, generator=g) * 2).to(DEV, torch.bfloat16)
    shifted = torch.empty(T, ncat + 8, device=DEV, dtype=torch.bfloat16)[:, 1:ncat + 1]
    shifted.copy_(proj)
    assert shifted.data_ptr() % 16 != 0
    pos = torch.randint(0, 4096, (T,), generator=g).to(DEV)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2).float() / D))
    ang = torch.arange(4096).float().view(-1, 1) * inv.view(1, -1)
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(DEV, tab_dtype), emb.sin().to(DEV, tab_dtype)
    vec = ops.proj_epilogue(dims, layout, proj, pos, cos, sin, has_g1)
    sca = ops.proj_epilogue(dims, layout, shifted, pos, cos, sin, has_g1)
    torch.cuda.synchronize()
    ops.check_device_error()
    for a, b in zip(vec, sca):
        if a is None:
            assert b is None
        else:
            assert torch.equal(a, b)
