"""Pins the CPU oracle (oracle/gsa_oracle.py) to outputs of the reference itself.

The golden fixtures were written by tests/golden/make_golden.py, which ran the unmodified
reference modules on the same seeded weights and inputs.  Every intermediate the oracle
restates must agree with them: bit for bit where the oracle performs the reference's own ops in
the same order, and as sets for the selected indices (compared over the mask-valid entries).
"""

import numpy as np
import pytest
import torch

from conftest import GOLDEN_NAMES, golden_inputs, load_golden
import gsa_oracle as O

torch.set_num_threads(max(1, torch.get_num_threads()))


def _sets(indices, mask):
    out = []
    for r in range(indices.shape[0]):
        out.append(np.sort(indices[r][mask[r].bool()].numpy().astype(np.int64)))
    return out


@pytest.fixture(scope="module", params=GOLDEN_NAMES)
def case(request):
    g, meta = load_golden(request.param)
    cfg, m, x = golden_inputs(meta)
    W = {k: v for k, v in m.state_dict().items()}
    ocfg = O.OracleConfig.from_config(cfg)
    L = x.shape[1]
    res = O.gsa_forward(W, ocfg, x, cos_cached=m.rotary_emb.cos_cached,
                        sin_cached=m.rotary_emb.sin_cached, chunk=64 if L <= 512 else 256,
                        keep=("q", "k", "v", "var", "k_values", "scores", "indices", "attn"))
    return request.param, g, meta, cfg, m, x, res


def test_weights_and_inputs_regenerate(case):
    name, g, meta, cfg, m, x, res = case
    sd = m.state_dict()
    for k, (s, ss, first) in meta["param_checksums"].items():
        t = sd[k].double()
        assert abs(float(t.sum()) - s) <= 1e-9 * max(1.0, abs(s)), k
        assert [float(v) for v in t.flatten()[:4]] == first, k
    xs = [float(x.double().sum()), float((x.double() ** 2).sum())]
    import json
    assert xs == json.loads(meta["x_checksum"])


def test_oracle_weight_init_regenerates_the_reference_parameters(case):
    """The oracle's own initialiser (no product module involved) gives the parameters whose
    checksums the reference recorded."""
    name, g, meta, cfg, m, x, res = case
    W = O.init_layer_weights(O.OracleConfig.from_config(cfg), int(meta["weight_seed"]), cfg.n_layers, x.dtype)
    assert set(W) == set(meta["param_checksums"])
    for k, (s, ss, first) in meta["param_checksums"].items():
        t = W[k].double()
        assert abs(float(t.sum()) - s) <= 1e-9 * max(1.0, abs(s)), k
        assert [float(v) for v in t.flatten()[:4]] == first, k


def test_projections_rope_g2(case):
    name, g, meta, cfg, m, x, res = case
    rows = g["rows"].long()
    assert torch.equal(res["q"][:, rows], g["q"])
    kk = res["k"] if g["k"].shape[1] == x.shape[1] else res["k"][:, rows]
    vv = res["v"] if g["v"].shape[1] == x.shape[1] else res["v"][:, rows]
    assert torch.equal(kk, g["k"])
    assert torch.equal(vv, g["v"])


def test_indexer_scores_chunked(case):
    name, g, meta, cfg, m, x, res = case
    rows = g["rows"].long()
    assert torch.equal(res["scores"][:, rows], g["scores"])


def test_variance_and_adaptive_k(case):
    name, g, meta, cfg, m, x, res = case
    assert torch.equal(res["var"], g["var"])
    assert torch.equal(res["k_values"].to(torch.int32), g["k_values"])


def test_selected_sets(case):
    name, g, meta, cfg, m, x, res = case
    rows = g["rows"].long()
    B = x.shape[0]
    for b in range(B):
        ours = _sets(res["indices"][b, rows], res["mask"][b, rows])
        ref = _sets(g["indices"][b], g["mask"][b])
        for a, r in zip(ours, ref):
            assert np.array_equal(a, r)


def test_stable_sets_match_reference(case):
    """The lower-index-first tie rule gives the reference's sets on these fixtures (no row has
    a tie at its k_t boundary)."""
    name, g, meta, cfg, m, x, res = case
    rows = g["rows"].long()
    for b in range(x.shape[0]):
        sc = g["scores"][b]
        kv = g["k_values"][b][rows] if cfg.use_adaptive_k else torch.full((len(rows),), min(cfg.k_base, x.shape[1]))
        ties = O.boundary_tie_rows(sc, kv)
        stable = O.topk_sets_stable(sc, kv)
        ref = _sets(g["indices"][b], g["mask"][b])
        for r, (a, rr) in enumerate(zip(stable, ref)):
            if r in ties:
                continue
            assert np.array_equal(a, rr), (name, b, r)


def test_attention_and_output(case):
    name, g, meta, cfg, m, x, res = case
    rows = g["rows"].long()
    assert torch.equal(res["attn"][:, rows], g["attn"])
    assert torch.equal(res["out"][:, rows], g["out"])


# ---- the selector's entropy and learned methods (adaptive_topk.py:104-133) ----
def _adaptive_golden():
    from pathlib import Path
    from safetensors.torch import load_file, safe_open
    path = Path(__file__).resolve().parent / "golden" / "adaptive_methods_b2_l96.safetensors"
    with safe_open(str(path), "pt") as f:
        meta = f.metadata()
    return load_file(str(path)), meta


@pytest.mark.parametrize("dname", ["float32", "bfloat16"])
@pytest.mark.parametrize("method", ["entropy", "learned"])
def test_adaptive_methods_match_the_reference(method, dname):
    import json
    t, meta = _adaptive_golden()
    temps = json.loads(meta["temperatures"])
    kb, kmin, kmax = int(meta["k_base"]), int(meta["k_min"]), int(meta["k_max"])
    scores = t[f"scores_{dname}"]
    pred = None
    if method == "learned":
        state = {k.split(".", 1)[1]: v.float() for k, v in t.items() if k.startswith(f"pred_{dname}.")}
        pred = O.adaptive_method_predictor(state, getattr(torch, dname))
    for j, temp in enumerate(temps):
        with torch.no_grad():
            k = O.adaptive_k_method(scores, method, kb, kmin, kmax, temp, pred)
        assert torch.equal(k.to(torch.int32), t[f"k_{method}_{dname}_t{j}"]), (method, dname, temp)
