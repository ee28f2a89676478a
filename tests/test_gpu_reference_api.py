"""The reference's own unit tests, restated against the drop-in (gsa_b200) on CUDA.

The reference ships three test files that define its module API contract (tests/test_attention.py,
tests/test_indexer.py, tests/test_gates.py).  Each test below makes the same calls with the same
shapes and configs and asserts what the reference's test asserts, with the modules and tensors on
the GPU (the drop-in has no CPU path).  Test names follow the reference's; every docstring cites
the test it restates.  ``test_adaptive_k_variation`` fails on the reference itself (early causal
rows have fewer valid keys than k_min, and k_t is clamped to the valid count,
adaptive_topk.py:132-136); it is kept as a strict expected failure, so the drop-in must fail it the
same way.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _cuda(cuda_ok):
    torch.manual_seed(0)


def _positions(B, L):
    return torch.arange(L, device=DEV).unsqueeze(0).expand(B, -1)


def _causal_scores(B, Lq, Lkv):
    s = torch.randn(B, Lq, Lkv, device=DEV)
    return s.masked_fill(torch.triu(torch.ones(Lq, Lkv, device=DEV), diagonal=1).bool(), float("-inf"))


# ---------------------------------------------------------------------------------------------
# tests/test_attention.py
# ---------------------------------------------------------------------------------------------
class TestGatedSparseAttention:
    @pytest.fixture
    def config(self):
        from gsa_b200 import GSAConfig

        return GSAConfig(d_model=512, n_heads=8, n_kv_heads=4, d_indexer=32, n_indexer_heads=2, k_base=64,
                         k_min=16, k_max=128, use_value_gate=True, use_output_gate=True, use_adaptive_k=True,
                         max_position_embeddings=2048)

    @pytest.fixture
    def gsa(self, config):
        from gsa_b200 import GatedSparseAttention

        return GatedSparseAttention(config).to(DEV)

    def test_initialization(self, gsa, config):
        """test_attention.py:44-56"""
        assert gsa.d_model == config.d_model
        assert gsa.n_heads == config.n_heads
        assert gsa.n_kv_heads == config.n_kv_heads
        assert gsa.q_proj.in_features == config.d_model
        assert gsa.q_proj.out_features == config.n_heads * config.d_head
        assert gsa.value_gate is not None
        assert gsa.output_gate is not None

    def test_forward_shape(self, gsa, config):
        """test_attention.py:58-66"""
        B, L = 2, 128
        x = torch.randn(B, L, config.d_model, device=DEV)
        output, _, _ = gsa(x, positions=_positions(B, L))
        assert output.shape == (B, L, config.d_model)

    def test_forward_with_cache(self, gsa, config):
        """test_attention.py:68-89"""
        B, L = 2, 64
        x = torch.randn(B, L, config.d_model, device=DEV)
        output1, cache, _ = gsa(x, positions=_positions(B, L), use_cache=True)
        assert cache is not None
        assert len(cache) == 2
        assert cache[0].shape[1] == L
        new = 16
        x2 = torch.randn(B, new, config.d_model, device=DEV)
        pos2 = torch.arange(L, L + new, device=DEV).unsqueeze(0).expand(B, -1)
        output2, cache2, _ = gsa(x2, positions=pos2, past_key_value=cache, use_cache=True)
        assert output2.shape == (B, new, config.d_model)
        assert cache2[0].shape[1] == L + new

    def test_gradient_flow(self, gsa, config):
        """test_attention.py:91-102"""
        B, L = 2, 64
        x = torch.randn(B, L, config.d_model, device=DEV, requires_grad=True)
        output, _, _ = gsa(x, positions=_positions(B, L))
        output.sum().backward()
        assert x.grad is not None
        assert not torch.isnan(x.grad).any()

    def test_causal_masking(self, gsa, config):
        """test_attention.py:104-114"""
        x = torch.randn(1, 32, config.d_model, device=DEV)
        output, _, attn_weights = gsa(x, positions=_positions(1, 32), output_attentions=True)
        assert output is not None

    def test_different_batch_sizes(self, gsa, config):
        """test_attention.py:116-124"""
        for B in [1, 4, 8]:
            x = torch.randn(B, 64, config.d_model, device=DEV)
            output, _, _ = gsa(x, positions=_positions(B, 64))
            assert output.shape == (B, 64, config.d_model)

    def test_different_seq_lengths(self, gsa, config):
        """test_attention.py:126-134"""
        for L in [32, 128, 256]:
            x = torch.randn(2, L, config.d_model, device=DEV)
            output, _, _ = gsa(x, positions=_positions(2, L))
            assert output.shape == (2, L, config.d_model)


class TestGSAWithoutGates:
    def test_no_gates(self):
        """test_attention.py:140-166"""
        from gsa_b200 import GSAConfig, GatedSparseAttention

        cfg = GSAConfig(d_model=512, n_heads=8, n_kv_heads=4, use_value_gate=False, use_output_gate=False)
        m = GatedSparseAttention(cfg).to(DEV)
        assert m.value_gate is None
        assert m.output_gate is None
        x = torch.randn(2, 64, cfg.d_model, device=DEV)
        output, _, _ = m(x, positions=_positions(2, 64))
        assert output.shape == (2, 64, cfg.d_model)


class TestGSACuda:
    @pytest.fixture
    def config(self):
        from gsa_b200 import GSAConfig

        return GSAConfig(d_model=512, n_heads=8, n_kv_heads=4)

    @pytest.fixture
    def gsa_cuda(self, config):
        from gsa_b200 import GatedSparseAttention

        return GatedSparseAttention(config).cuda()

    def test_cuda_forward(self, gsa_cuda, config):
        """test_attention.py:181-189"""
        x = torch.randn(2, 128, config.d_model, device="cuda")
        output, _, _ = gsa_cuda(x, positions=_positions(2, 128))
        assert output.device.type == "cuda"
        assert output.shape == (2, 128, config.d_model)

    def test_mixed_precision(self, gsa_cuda, config):
        """test_attention.py:191-202"""
        x = torch.randn(2, 128, config.d_model, device="cuda", dtype=torch.bfloat16)
        gsa_cuda = gsa_cuda.to(torch.bfloat16)
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            output, _, _ = gsa_cuda(x, positions=_positions(2, 128))
        assert output.dtype == torch.bfloat16


# ---------------------------------------------------------------------------------------------
# tests/test_indexer.py
# ---------------------------------------------------------------------------------------------
class TestGatedLightningIndexer:
    @pytest.fixture
    def indexer(self):
        from gsa_b200 import GatedLightningIndexer

        return GatedLightningIndexer(d_model=512, d_indexer=32, n_indexer_heads=4, activation="sigmoid").to(DEV)

    def test_initialization(self, indexer):
        """test_indexer.py:27-32"""
        assert indexer.d_model == 512
        assert indexer.d_indexer == 32
        assert indexer.n_indexer_heads == 4
        assert indexer.activation == "sigmoid"

    def test_forward_shape(self, indexer):
        """test_indexer.py:34-44"""
        scores = indexer(torch.randn(2, 64, 512, device=DEV), _positions(2, 64))
        assert scores.shape == (2, 64, 64)

    def test_causal_masking(self, indexer):
        """test_indexer.py:46-58"""
        scores = indexer(torch.randn(1, 32, 512, device=DEV), _positions(1, 32)).cpu()
        for i in range(32):
            for j in range(i + 1, 32):
                assert scores[0, i, j] == float("-inf")

    def test_sigmoid_bounded_scores(self, indexer):
        """test_indexer.py:60-73"""
        scores = indexer(torch.randn(2, 32, 512, device=DEV), _positions(2, 32))
        valid = scores[scores != float("-inf")]
        assert (valid >= 0).all()
        assert (valid <= indexer.n_indexer_heads + 1).all()

    def test_relu_activation(self):
        """test_indexer.py:75-91"""
        from gsa_b200 import GatedLightningIndexer

        ix = GatedLightningIndexer(d_model=512, d_indexer=32, n_indexer_heads=4, activation="relu").to(DEV)
        scores = ix(torch.randn(2, 32, 512, device=DEV), _positions(2, 32))
        assert (scores[scores != float("-inf")] >= 0).all()

    def test_gradient_flow(self, indexer):
        """test_indexer.py:93-106"""
        h = torch.randn(2, 32, 512, device=DEV, requires_grad=True)
        scores = indexer(h, _positions(2, 32))
        scores[scores != float("-inf")].sum().backward()
        assert h.grad is not None
        assert not torch.isnan(h.grad).any()

    def test_cross_attention(self, indexer):
        """test_indexer.py:108-127"""
        from gsa_b200 import GatedLightningIndexer

        ix = GatedLightningIndexer(d_model=512, d_indexer=32, n_indexer_heads=4, use_causal_mask=False).to(DEV)
        scores = ix(torch.randn(2, 32, 512, device=DEV), _positions(2, 32),
                    kv_hidden_states=torch.randn(2, 64, 512, device=DEV))
        assert scores.shape == (2, 32, 64)


class TestAdaptiveTopKSelector:
    @pytest.fixture
    def selector(self):
        from gsa_b200 import AdaptiveTopKSelector

        return AdaptiveTopKSelector(k_base=32, k_min=8, k_max=64, use_adaptive=True, temperature=1.0)

    @pytest.fixture
    def selector_fixed(self):
        from gsa_b200 import AdaptiveTopKSelector

        return AdaptiveTopKSelector(k_base=32, k_min=8, k_max=64, use_adaptive=False)

    def test_initialization(self, selector):
        """test_indexer.py:152-157"""
        assert selector.k_base == 32
        assert selector.k_min == 8
        assert selector.k_max == 64
        assert selector.use_adaptive is True

    def test_forward_shape(self, selector):
        """test_indexer.py:159-178"""
        indices, mask = selector(_causal_scores(2, 64, 64), 64, 64)
        assert indices.shape[0] == 2 and indices.shape[1] == 64 and indices.shape[2] <= selector.k_max
        assert mask.shape == indices.shape

    def test_fixed_k(self, selector_fixed):
        """test_indexer.py:180-190"""
        indices, mask = selector_fixed(_causal_scores(2, 64, 64), 64, 64)
        assert indices.shape[2] == min(selector_fixed.k_base, 64)

    @pytest.mark.xfail(strict=True, raises=AssertionError, reason="fails on the reference too: k_t is clamped to the row's valid "
                                           "count, which is below k_min for the first causal rows")
    def test_adaptive_k_variation(self, selector):
        """test_indexer.py:192-207"""
        indices, mask, k_values = selector(_causal_scores(4, 64, 64), 64, 64, return_k_values=True)
        assert k_values is not None
        assert (k_values >= selector.k_min).all()
        assert (k_values <= selector.k_max).all()

    def test_mask_validity(self, selector):
        """test_indexer.py:209-225"""
        indices, mask = selector(_causal_scores(2, 32, 32), 32, 32)
        for b in range(2):
            for q in range(32):
                n = mask[b, q].sum().item()
                assert 0 <= n <= selector.k_max

    def test_indices_in_range(self, selector):
        """test_indexer.py:227-239"""
        indices, mask = selector(_causal_scores(2, 64, 64), 64, 64)
        assert (indices >= 0).all()
        assert (indices < 64).all()


class TestIndexerIntegration:
    def test_indexer_to_selector_pipeline(self):
        """test_indexer.py:245-277"""
        from gsa_b200 import AdaptiveTopKSelector, GatedLightningIndexer

        ix = GatedLightningIndexer(d_model=512, d_indexer=32, n_indexer_heads=4).to(DEV)
        sel = AdaptiveTopKSelector(k_base=16, k_min=4, k_max=32, use_adaptive=True)
        scores = ix(torch.randn(2, 64, 512, device=DEV), _positions(2, 64))
        indices, mask = sel(scores, 64, 64)
        assert scores.shape == (2, 64, 64)
        assert indices.shape[0] == 2 and indices.shape[1] == 64
        assert mask.shape == indices.shape


# ---------------------------------------------------------------------------------------------
# tests/test_gates.py
# ---------------------------------------------------------------------------------------------
class TestValueGate:
    @pytest.fixture
    def value_gate(self):
        from gsa_b200 import ValueGate

        return ValueGate(d_model=512, n_kv_heads=8, d_head=64, bias_init=0.5).to(DEV)

    def test_initialization(self, value_gate):
        """test_gates.py:26-39"""
        assert value_gate.d_model == 512 and value_gate.n_kv_heads == 8 and value_gate.d_head == 64
        b = value_gate.gate_proj.bias
        assert b is not None
        assert torch.allclose(b, torch.full_like(b, 0.5), atol=1e-6)

    def test_forward_shape(self, value_gate):
        """test_gates.py:41-51"""
        v = torch.randn(2, 64, 8, 64, device=DEV)
        assert value_gate(v, torch.randn(2, 64, 512, device=DEV)).shape == v.shape

    def test_gating_bounds(self, value_gate):
        """test_gates.py:53-69"""
        v = torch.randn(2, 64, 8, 64, device=DEV)
        value_gate.eval()
        value_gate(v, torch.randn(2, 64, 512, device=DEV))
        assert value_gate.last_gate_scores is not None
        assert (value_gate.last_gate_scores >= 0).all()
        assert (value_gate.last_gate_scores <= 1).all()

    def test_gradient_flow(self, value_gate):
        """test_gates.py:71-86"""
        v = torch.randn(2, 32, 8, 64, device=DEV, requires_grad=True)
        h = torch.randn(2, 32, 512, device=DEV, requires_grad=True)
        value_gate(v, h).sum().backward()
        assert v.grad is not None and h.grad is not None
        assert not torch.isnan(v.grad).any() and not torch.isnan(h.grad).any()

    def test_statistics(self, value_gate):
        """test_gates.py:88-106"""
        value_gate.eval()
        value_gate(torch.randn(2, 64, 8, 64, device=DEV), torch.randn(2, 64, 512, device=DEV))
        stats = value_gate.get_gate_statistics()
        for key in ("mean", "std", "min", "max"):
            assert key in stats
        assert 0 <= stats["mean"] <= 1


class TestOutputGate:
    @pytest.fixture
    def output_gate(self):
        from gsa_b200 import OutputGate

        return OutputGate(d_model=512, n_heads=8, d_head=64, bias_init=0.5, per_head=True).to(DEV)

    def test_initialization(self, output_gate):
        """test_gates.py:124-129"""
        assert output_gate.d_model == 512 and output_gate.n_heads == 8 and output_gate.d_head == 64
        assert output_gate.per_head is True

    def test_forward_shape(self, output_gate):
        """test_gates.py:131-141"""
        a = torch.randn(2, 64, 8, 64, device=DEV)
        assert output_gate(a, torch.randn(2, 64, 512, device=DEV)).shape == a.shape

    def test_per_head_vs_scalar(self):
        """test_gates.py:143-162"""
        from gsa_b200 import OutputGate

        per_head = OutputGate(512, 8, 64, per_head=True).to(DEV)
        scalar = OutputGate(512, 8, 64, per_head=False).to(DEV)
        a = torch.randn(2, 32, 8, 64, device=DEV)
        h = torch.randn(2, 32, 512, device=DEV)
        assert per_head(a, h).shape == scalar(a, h).shape
        assert per_head.gate_proj.out_features == 8 * 64
        assert scalar.gate_proj.out_features == 8

    def test_gradient_flow(self, output_gate):
        """test_gates.py:164-177"""
        a = torch.randn(2, 32, 8, 64, device=DEV, requires_grad=True)
        h = torch.randn(2, 32, 512, device=DEV, requires_grad=True)
        output_gate(a, h).sum().backward()
        assert a.grad is not None and h.grad is not None


class TestGateCombinations:
    @pytest.mark.parametrize("use_v,use_o", [(True, True), (True, False), (False, True)])
    def test_gate_combinations(self, use_v, use_o):
        """test_gates.py:183-229 (test_both_gates, test_only_value_gate, test_only_output_gate)"""
        from gsa_b200 import GSAConfig, GatedSparseAttention

        cfg = GSAConfig(d_model=256, n_heads=4, n_kv_heads=2, use_value_gate=use_v, use_output_gate=use_o)
        m = GatedSparseAttention(cfg).to(DEV)
        assert (m.value_gate is not None) == use_v
        assert (m.output_gate is not None) == use_o
        out, _, _ = m(torch.randn(1, 48, 256, device=DEV))
        assert out.shape == (1, 48, 256)
