"""generate()'s sampling against the reference's generate (gsa_llama.py:344-430).

The fixture ``tests/golden/sampling_b3_v96.safetensors`` was written by running the reference's
``GSALlamaForCausalLM.generate`` with its forward replaced by seeded logits (quantised, so ties
occur at the top-k and top-p cuts) under ``torch.manual_seed(seed)``, for several (temperature,
top_k, top_p, do_sample) settings.  ``decode_loop`` -- the token loop of our generate, with the
filter as one function -- fed the same logits under the same seed must pick the same tokens: its
filtered distributions equal the reference's bit for bit, so torch.multinomial draws the same
samples.  CPU only: the loop is host code around the model's step."""

import json

import torch

from conftest import GOLDEN


def _fixture():
    from safetensors import safe_open

    with safe_open(str(GOLDEN / "sampling_b3_v96.safetensors"), "pt") as f:
        meta = dict(f.metadata())
        t = {k: f.get_tensor(k) for k in f.keys()}
    return t, json.loads(meta["settings"]), int(meta["steps"])


def test_decode_loop_samples_the_reference_tokens():
    from gsa_b200.models import decode_loop

    t, settings, steps = _fixture()
    prompt = t["prompt"].long()
    for j, (temp, top_k, top_p, do_sample, seed) in enumerate(settings):
        fed = []

        def step(tokens, first):
            fed.append((int(tokens.shape[1]), first))
            return t["logits"][len(fed) - 1][:, -1, :].clone()

        torch.manual_seed(seed)
        out = decode_loop(step, prompt, steps, temp, top_k, top_p, do_sample, None)
        assert fed == [(prompt.shape[1], True)] + [(1, False)] * (steps - 1)
        assert torch.equal(out, t[f"tokens{j}"].long()), (j, temp, top_k, top_p, do_sample)


def test_filter_keeps_the_most_likely_token_and_ties_at_the_top_k_cut():
    from gsa_b200.models import filter_logits

    logits = torch.tensor([[3.0, 1.0, 1.0, 1.0, 0.5, -2.0]])
    out = filter_logits(logits, top_k=2)
    # the second-largest value is tied three ways: all three stay
    assert torch.isfinite(out).tolist() == [[True, True, True, True, False, False]]
    out = filter_logits(logits, top_p=0.01)
    assert torch.isfinite(out).tolist() == [[True, False, False, False, False, False]]
    out = filter_logits(logits, temperature=2.0)
    assert torch.allclose(out, logits / 2)


def test_eos_stops_the_loop():
    from gsa_b200.models import decode_loop

    V = 8
    logits = torch.full((2, V), -10.0)
    logits[:, 3] = 10.0

    def step(tokens, first):
        return logits.clone()

    out = decode_loop(step, torch.zeros(2, 4, dtype=torch.long), 10, 1.0, 0, 1.0, False, eos_token_id=3)
    assert out.shape == (2, 5) and bool((out[:, -1] == 3).all())
