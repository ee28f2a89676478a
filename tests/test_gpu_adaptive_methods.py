"""The selector's entropy and learned adaptive-k methods on the GPU (adaptive_topk.py:104-133):
the native row-summary pass (gsa_row_summary) feeds the module's k computation.  Against the
reference's own k_t (golden fixture written by tests/golden/make_golden.py) and against the
oracle on a longer random case.

k_t truncates a float (adaptive_topk.py:133), and the row statistics sum in a different order than
torch's CPU kernels (the softmax normaliser, the entropy and the moments), so a k_t may land one
below or above the reference's where its float value sits on an integer: |dk| <= 1 everywhere
(one bf16 step of k for the learned method in bf16, whose k is a bf16 value) and at least 95% of
the rows equal.  The statistics themselves: within 2 units in the last place of
the dtype (entropy, std) or exact (count, max)."""

import json
from pathlib import Path

import pytest
import torch
from safetensors.torch import load_file, safe_open

import gsa_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden" / "adaptive_methods_b2_l96.safetensors"


def _golden():
    with safe_open(str(GOLDEN), "pt") as f:
        meta = f.metadata()
    return load_file(str(GOLDEN)), meta


def _selector(method, dname, t, kb, kmin, kmax, temp):
    from gsa_b200.attention import AdaptiveTopKSelector

    dt = getattr(torch, dname)
    sel = AdaptiveTopKSelector(k_base=kb, k_min=kmin, k_max=kmax, use_adaptive=True, temperature=temp,
                               adaptive_method=method)
    if method == "learned":
        state = {k.split(".", 1)[1]: v.float() for k, v in t.items() if k.startswith(f"pred_{dname}.")}
        sel.k_predictor.load_state_dict(state)
    return sel.to(dt).to(DEV)


def _check_k(k, ref, what, rel=0.0):
    """|dk| <= max(1, rel * k_ref) everywhere, >= 95% of the rows equal.  The learned method in
    bf16 forms k = k_min + k_scale (k_max - k_min) in bf16 (adaptive_topk.py:127), so a one-ulp
    difference of k_scale moves k by one bf16 step of its magnitude: rel = 2^-7 there."""
    d = (k.long().cpu() - ref.long()).abs()
    tol = torch.clamp((ref.long().abs().double() * rel).ceil().long(), min=1)
    assert bool((d <= tol).all()), (what, int(d.max()))
    assert float((d == 0).double().mean()) >= 0.95, (what, float((d == 0).double().mean()))


@pytest.mark.parametrize("dname", ["float32", "bfloat16"])
@pytest.mark.parametrize("method", ["entropy", "learned"])
def test_adaptive_methods_against_the_reference(cuda_ok, method, dname):
    from gsa_b200 import ops

    t, meta = _golden()
    temps = json.loads(meta["temperatures"])
    kb, kmin, kmax = int(meta["k_base"]), int(meta["k_min"]), int(meta["k_max"])
    scores = t[f"scores_{dname}"]
    B, L, _ = scores.shape
    for j, temp in enumerate(temps):
        sel = _selector(method, dname, t, kb, kmin, kmax, temp)
        with torch.no_grad():
            idx, mask, k = sel(scores.to(DEV), L, L, return_k_values=True)
        torch.cuda.synchronize()
        ops.check_device_error()
        _check_k(k, t[f"k_{method}_{dname}_t{j}"], (method, dname, temp),
                 2.0 ** -7 if (method, dname) == ("learned", "bfloat16") else 0.0)
        # the mask keeps k_t of each row's candidates
        assert torch.equal(mask.sum(-1).cpu(), k.cpu().to(mask.sum(-1).dtype))


@pytest.mark.parametrize("dname", ["float32", "bfloat16"])
def test_row_summary_statistics(cuda_ok, dname):
    """The native statistics against the reference's torch ops on the same scores (CPU): 2048 random
    rows of 2048 columns, causal mask, values spread like indexer scores."""
    from gsa_b200 import ops

    dt = getattr(torch, dname)
    L = 2048
    g = torch.Generator().manual_seed(3)
    s = (torch.rand(1, L, L, generator=g) * 4).masked_fill(torch.triu(torch.ones(L, L, dtype=torch.bool), 1),
                                                        float("-inf")).to(dt)
    summ = ops.row_summary(s[0].to(DEV), dt).cpu()
    valid = s[0] != float("-inf")
    masked = s[0].masked_fill(~valid, 0)
    probs = torch.softmax(s[0].float(), dim=-1).to(dt).masked_fill(~valid, 0)
    ent = -(probs * torch.log(probs + 1e-10)).sum(-1)
    ref = {"count": valid.sum(-1).float(), "mean": masked.mean(-1).float(), "std": masked.std(-1).float(),
           "max": masked.max(-1).values.float(), "entropy": ent.float()}
    ulp = 2.0 ** -7 if dt == torch.bfloat16 else 2.0 ** -22
    assert torch.equal(summ[:, 0], ref["count"])
    assert torch.equal(summ[:, 3], ref["max"])
    for col, name in ((1, "mean"), (2, "std"), (4, "entropy")):
        rel = ((summ[:, col] - ref[name]).abs() / ref[name].abs().clamp_min(1e-30)).max()
        assert float(rel) <= 2 * ulp, (name, float(rel))


def test_adaptive_methods_against_the_oracle_2048(cuda_ok):
    """A longer case (2 x 2048 rows) for both methods in bf16: k_t vs the oracle's torch ops run on
    the same GPU, so that the learned method's predictor (a bf16 Linear, whose rounding differs
    between the CPU and the GPU GEMM) is the same computation on both sides and only the native row
    statistics are under test."""
    t, _ = _golden()
    L = 2048
    g = torch.Generator().manual_seed(4)
    s = (torch.rand(2, L, L, generator=g) * 3).masked_fill(torch.triu(torch.ones(L, L, dtype=torch.bool), 1),
                                                        float("-inf")).to(torch.bfloat16)
    for method in ("entropy", "learned"):
        sel = _selector(method, "bfloat16", t, 512, 128, 1024, 0.8)
        with torch.no_grad():
            _, _, k = sel(s.to(DEV), L, L, return_k_values=True)
            pred = None
            if method == "learned":
                state = {k2.split(".", 1)[1]: v.float() for k2, v in t.items() if k2.startswith("pred_bfloat16.")}
                pred = O.adaptive_method_predictor(state, torch.bfloat16).to(DEV)
            ref = O.adaptive_k_method(s.to(DEV), method, 512, 128, 1024, 0.8, pred).cpu()
        _check_k(k, ref, method, 2.0 ** -7 if method == "learned" else 0.0)
