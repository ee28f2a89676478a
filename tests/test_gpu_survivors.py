"""The threshold-survivor candidate pass (gsa_indexer_survivors) against the exact one
(gsa_indexer_select) on the same inputs: each row's survivors are in ascending column order,
contain its k_eff best keys, and the final selection (gsa_select_finalize) from them equals the
selection from the exact candidates.  Covered: rows short enough to keep every key, thresholded
rows, batch > 1 with a query offset, non-causal rows, H_I = 4, the fp32 indexer, tied
scores that defeat the threshold so that the exact per-row selection takes over, and decode
rows (one or two per sequence, many sequences per pass: the few-row compaction)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(B, Lq, Lkv, HI, seed, dtype=torch.bfloat16, dI=64, zero_keys_from=None):
    g = torch.Generator().manual_seed(seed)
    qI = (torch.randn(B, Lq, HI * dI, generator=g) * 1.3).to(dtype)
    kI = torch.randn(B, Lkv, dI, generator=g) * 1.4
    if zero_keys_from is not None:
        kI[:, zero_keys_from:] = 0.0     # identical keys: their scores tie within each row
    kI = kI.to(dtype)
    w = torch.sigmoid(torch.randn(B * Lq, HI, generator=g) * 0.3)
    bias = torch.randn(HI, generator=g) * 0.1
    shift = 0.5 * w.sum(-1)
    return [t.to(DEV) for t in (qI, kI, w, bias, shift)]


@pytest.mark.parametrize("dtype,B,Lq,Lkv,HI,q_pos0,causal,k_eff,zero_from,chunk", [
    (torch.bfloat16, 1, 12000, 12000, 8, 0, True, 4096, None, 5000),   # short rows keep every key
    (torch.bfloat16, 2, 600, 30000, 8, 29400, True, 2048, None, 256),  # batch > 1, offset-causal
    (torch.bfloat16, 1, 300, 20000, 4, 0, False, 1024, None, 300),     # non-causal, H_I = 4
    (torch.float32, 1, 400, 12000, 8, 11600, True, 1024, None, 128),   # fp32 indexer kernel
    (torch.bfloat16, 1, 256, 20000, 8, 19744, True, 4096, 0, 100),     # all keys tie: exact fallback
    (torch.bfloat16, 1, 512, 24000, 8, 23488, True, 4096, 12000, 512), # half the keys tie
    (torch.bfloat16, 37, 1, 30000, 8, 29999, True, 4096, None, 64),   # decode rows: few-row compaction
    (torch.bfloat16, 20, 1, 20000, 8, 19999, True, 4096, 0, 64),      # decode rows, all tie: exact fallback
    (torch.bfloat16, 9, 2, 9000, 4, 8998, True, 2048, None, 64),      # two tokens per sequence, H_I = 4
])
def test_survivors_select_the_exact_keys(cuda_ok, dtype, B, Lq, Lkv, HI, q_pos0, causal, k_eff, zero_from,
                                         chunk):
    from gsa_b200 import ops

    dI = 64
    dims = ops.make_dims(4096, 32, 8, 128, HI, dI)
    qI, kI, w, bias, shift = _inputs(B, Lq, Lkv, HI, seed=Lkv + HI, dtype=dtype, zero_keys_from=zero_from)
    R = B * Lq
    scale = 1 / math.sqrt(dI)
    t = torch.arange(R) % Lq
    n = torch.clamp(t + q_pos0 + 1, max=Lkv) if causal else torch.full((R,), Lkv)
    g = torch.Generator().manual_seed(5)
    kt = torch.minimum(torch.randint(1, k_eff + 1, (R,), generator=g), n).int()
    kt[::7] = torch.minimum(torch.tensor(k_eff), n[::7]).int()
    kt = kt.to(DEV)

    ci, cs, cc, st = ops.indexer_select(dims, qI, kI, w, bias, scale, shift, k_eff, q_pos0=q_pos0,
                                        causal=causal, chunk_rows=chunk)
    ref_sel, ref_cnt, _ = ops.select_finalize(ci, cs, cc, kt, sel_ld=k_eff)
    si, ss, sc, st2 = ops.indexer_survivors(dims, qI, kI, w, bias, scale, shift, k_eff, q_pos0=q_pos0,
                                            causal=causal, chunk_rows=chunk)
    sel, cnt, _ = ops.select_finalize(si, ss, sc, kt, sel_ld=k_eff)
    torch.cuda.synchronize()
    ops.check_device_error()

    assert torch.equal(cnt, ref_cnt)
    valid = torch.arange(k_eff, device=DEV).view(1, -1) < ref_cnt.view(-1, 1)
    assert torch.equal(sel[valid], ref_sel[valid])
    assert torch.equal(st2[:, 2], st[:, 2])
    # survivors: ascending columns, within [min(k_eff, n), cap], a superset of the exact candidates
    sc_c, cc_c = sc.cpu(), cc.cpu()
    assert bool((sc_c <= ops.SURVIVOR_CAP).all()) and bool((sc_c >= torch.clamp(n, max=k_eff)).all())
    si_c, ci_c = si.cpu(), ci.cpu()
    for r in list(range(0, R, max(1, R // 40))) + [R - 1]:
        s_row = si_c[r, :int(sc_c[r])]
        assert bool((s_row[1:] > s_row[:-1]).all()), r
        e_row = ci_c[r, :int(cc_c[r])]
        assert bool(torch.isin(e_row, s_row).all()), r


def test_layer_candidate_paths_agree(cuda_ok):
    """A bf16 layer forward with threshold survivors equals the exact-candidate forward bit for bit."""
    from gsa_b200 import GatedSparseAttention, GSAConfig

    cfg = GSAConfig(d_model=1024, n_heads=8, n_kv_heads=2, d_indexer=64, n_indexer_heads=8, k_base=2048,
                    k_min=256, k_max=4096, max_position_embeddings=16384)
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).to(DEV).to(torch.bfloat16).eval()
    x = torch.randn(1, 10000, 1024, generator=torch.Generator().manual_seed(1)).to(DEV, torch.bfloat16)
    cap_s, cap_e = {}, {}
    with torch.no_grad():
        out_s = m._forward_impl(x, None, None, False, False, capture=cap_s)[0]
        m.selection_path = "exact"
        out_e = m._forward_impl(x, None, None, False, False, capture=cap_e)[0]
        m.selection_path = "auto"
    torch.cuda.synchronize()
    assert cap_s["candidate_path"] == "survivors" and cap_e["candidate_path"] == "exact"
    assert torch.equal(cap_s["cnt"], cap_e["cnt"])
    assert torch.equal(out_s, out_e)


def test_layer_forward_is_deterministic(cuda_ok):
    """Repeated bf16 forwards give bit-identical outputs: no shared-memory slot is refilled while a
    read of it is still in flight (compaction ring, SDPA ring), and fp64 statistic sums that
    differ in their last bits do not change the selection."""
    from gsa_b200 import GatedSparseAttention, GSAConfig

    cfg = GSAConfig(d_model=1024, n_heads=8, n_kv_heads=2, d_indexer=64, n_indexer_heads=8, k_base=2048,
                    k_min=256, k_max=4096, max_position_embeddings=16384)
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).to(DEV).to(torch.bfloat16).eval()
    x = torch.randn(1, 10000, 1024, generator=torch.Generator().manual_seed(1)).to(DEV, torch.bfloat16)
    with torch.no_grad():
        outs = [m(x)[0] for _ in range(6)]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
