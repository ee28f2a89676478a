"""Host-side pieces of the layer's backward, on CPU tensors: the transpose of RoPE
(rope.py:151-185) and the gate activations' derivatives (value_gate.py:98-106,
output_gate.py:111-119) against torch autograd of the oracle's forward formulas."""

import pytest
import torch

import gsa_oracle as O


def test_rope_backward_is_the_transpose_of_rope():
    from gsa_b200.attention import _rope_backward

    g = torch.Generator().manual_seed(0)
    T, Hh, D = 37, 3, 64
    cos, sin = O.rope_cache(D, 128, 10000.0, None)
    pos = torch.randint(0, 128, (T,), generator=g)
    c, s = cos[pos], sin[pos]
    x = torch.randn(T, Hh, D, generator=g, dtype=torch.float64).requires_grad_(True)
    dy = torch.randn(T, Hh, D, generator=g, dtype=torch.float64)
    y = O.apply_rope(x.unsqueeze(0), c.double().unsqueeze(0), s.double().unsqueeze(0))[0]
    (y * dy).sum().backward()
    ours = _rope_backward(dy.float(), c, s).double()
    assert torch.allclose(ours, x.grad, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("act", ["sigmoid", "tanh", "silu"])
def test_gate_activation_and_derivative(act):
    from gsa_b200.attention import _act, _act_grad

    x = torch.linspace(-9, 9, 1001, dtype=torch.float64).requires_grad_(True)
    y = O.gate_activation(x, act)
    y.sum().backward()
    assert torch.allclose(_act(x.detach(), act).double(), y.detach(), rtol=1e-6, atol=1e-7)
    assert torch.allclose(_act_grad(x.detach(), act).double(), x.grad, rtol=1e-5, atol=1e-7)
