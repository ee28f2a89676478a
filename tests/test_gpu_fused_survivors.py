"""The fused survivor pass (gsa_indexer_survivors_fused: the tensor-core indexer writes each row's
survivors itself, no score matrix in HBM) against the materialised one (gsa_indexer_survivors:
every score to a scratch, then the streaming compaction) on the same inputs:

* the row statistics are bit-identical (same epilogue arithmetic, same summation order);
* every candidate's score equals the materialised score of its column, bit for bit, and each
  row's candidates are ascending, unique and causal;
* the final selection (gsa_select_finalize) from the two candidate sets is identical for random
  k_t, k_t = k_eff included -- both sets hold every score at or above a threshold below the row's
  k_eff-th best, so the same k_t best with the same lower-column-first ties.

Cases: thresholded rows over several chunks; two sequences in one chunk; a query offset; rows
short enough to keep every key; non-causal rows; and planted keys whose sampled statistics mislead the threshold
(too many survivors, too few, one key range holding more than its segment's room), so that rows
fall back to the exact selection from their recomputed query block -- the test reads the failed-
row count to make sure they did.  The gated indexer scores are gated_indexer.py:114-153; the
candidate stage adaptive_topk.py:138-177."""

import ctypes as C
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
K_EFF = 4096


def _inputs(B, Lq, Lkv, seed, plant=None):
    g = torch.Generator().manual_seed(seed)
    HI, dI = 8, 64
    qI = (torch.randn(B, Lq, HI * dI, generator=g) * 1.3)
    kI = torch.randn(B, Lkv, dI, generator=g) * 1.4
    if plant == "unsampled_tie":
        # keys of the tiles the sampled pass skips (tile % 16 != 0) are all zero: their scores tie
        tiles = torch.arange(Lkv) // 128
        kI[:, tiles % 16 != 0] = 0.0
    elif plant == "one_range":
        # every key zero but those of one 4096-key range, which are one repeated vector: the
        # range's keys tie, above or below the rest, and take the row's top k_eff together
        kI.zero_()
        kI[:, 8192:12288] = 3.0 * torch.randn(dI, generator=g)
    g2 = torch.Generator().manual_seed(seed + 1)
    w = torch.sigmoid(torch.randn(B * Lq, HI, generator=g2) * 0.3)
    bias = torch.randn(HI, generator=g2) * 0.1
    shift = 0.5 * w.sum(-1)
    return [t.to(DEV) for t in (qI.to(torch.bfloat16), kI.to(torch.bfloat16), w, bias, shift)]


def _fused_fail_count(ops, dims, qI, kI, w, bias, scale, shift, q_pos0, chunk):
    """One direct call of gsa_indexer_survivors_fused with its workspace at hand: the failed rows
    of the last chunk (read from the workspace after the call)."""
    from gsa_b200 import _lib

    lib = _lib.lib()
    B, Lq, _ = qI.shape
    Lkv = kI.shape[1]
    R = B * Lq
    cap = ops.SURVIVOR_CAP
    ws_bytes = lib.gsa_survivors_fused_workspace_size(chunk, Lkv, K_EFF, cap)
    ws = torch.zeros(ws_bytes, device=DEV, dtype=torch.uint8)
    ci = torch.empty(R, cap, device=DEV, dtype=torch.int32)
    cs = torch.empty(R, cap, device=DEV, dtype=torch.float32)
    cc = torch.empty(R, device=DEV, dtype=torch.int32)
    st = torch.zeros(R, 3, device=DEV, dtype=torch.float64)
    wf = w.reshape(R, -1).float().contiguous()
    _lib.call("gsa_indexer_survivors_fused", C.byref(dims), 1, B, Lq, Lkv, q_pos0, 1,
              qI.data_ptr(), qI.stride(1), qI.stride(0), kI.data_ptr(), kI.stride(1), kI.stride(0),
              wf.data_ptr(), bias.data_ptr(), float(scale), shift.data_ptr(), K_EFF, cap,
              ci.data_ptr(), cs.data_ptr(), cc.data_ptr(), st.data_ptr(), chunk, ws.data_ptr(), ws_bytes,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    a256 = lambda x: (x + 255) // 256 * 256
    off = a256(lib.gsa_workspace_size(chunk, Lkv)) + a256(chunk * 4)
    return int(ws[off:off + 4].view(torch.int32).item())


@pytest.mark.parametrize("B,Lq,Lkv,q_pos0,chunk,plant,causal", [
    (1, 20000, 20000, 0, 6000, None, True),            # thresholded rows over four chunks
    (2, 9000, 9000, 0, 18000, None, True),             # two sequences in one chunk; most rows keep every key
    (1, 3000, 40000, 37000, 3000, None, True),         # query offset: long rows only
    (2, 700, 30000, 0, 500, None, False),              # non-causal rows, two sequences in 500-row chunks
    (1, 2048, 20000, 17952, 2048, "unsampled_tie", True),  # sampled statistics miss the tied keys
    (1, 1024, 100000, 98976, 1024, "one_range", True),  # one range holds the top k_eff: segment overflow
])
def test_fused_survivors_match_materialised(cuda_ok, B, Lq, Lkv, q_pos0, chunk, plant, causal):
    from gsa_b200 import ops

    dims = ops.make_dims(4096, 32, 8, 128, 8, 64)
    qI, kI, w, bias, shift = _inputs(B, Lq, Lkv, seed=Lkv + Lq, plant=plant)
    R = B * Lq
    scale = 1 / math.sqrt(64)
    t = torch.arange(R) % Lq
    n = torch.clamp(t + q_pos0 + 1, max=Lkv) if causal else torch.full((R,), Lkv)
    g = torch.Generator().manual_seed(7)
    kt = torch.minimum(torch.randint(1, K_EFF + 1, (R,), generator=g), n).int()
    kt[::5] = torch.minimum(torch.tensor(K_EFF), n[::5]).int()
    kt = kt.to(DEV)

    mi, ms, mc, mst = ops.indexer_survivors(dims, qI, kI, w, bias, scale, shift, K_EFF, q_pos0=q_pos0,
                                            causal=causal, chunk_rows=chunk, fused=False)
    assert ops.last_survivor_path == "materialised"
    fi, fs, fc, fst = ops.indexer_survivors(dims, qI, kI, w, bias, scale, shift, K_EFF, q_pos0=q_pos0,
                                            causal=causal, chunk_rows=chunk, fused=True)
    assert ops.last_survivor_path == "fused"
    m_sel, m_cnt, _ = ops.select_finalize(mi, ms, mc, kt, sel_ld=K_EFF)
    f_sel, f_cnt, _ = ops.select_finalize(fi, fs, fc, kt, sel_ld=K_EFF)
    torch.cuda.synchronize()
    ops.check_device_error()

    assert torch.equal(fst, mst)
    assert torch.equal(f_cnt, m_cnt)
    valid = torch.arange(K_EFF, device=DEV).view(1, -1) < m_cnt.view(-1, 1)
    assert torch.equal(f_sel[valid], m_sel[valid])
    fc_c = fc.cpu()
    assert bool((fc_c <= ops.SURVIVOR_CAP).all()) and bool((fc_c >= torch.clamp(n, max=K_EFF)).all())

    # candidate scores against the materialised scores of the same columns, sampled rows
    rows = sorted(set(list(range(0, R, max(1, R // 24))) + [R - 1]))
    fi_c, fs_c = fi.cpu(), fs.cpu()
    for r in rows:
        b, tt = divmod(r, Lq)
        sc = ops.indexer_scores(dims, qI[b:b + 1, tt:tt + 1], kI[b:b + 1], w.view(B, Lq, -1)[b:b + 1, tt:tt + 1],
                                bias, scale, q_pos0=q_pos0 + tt, causal=causal)[0].cpu()
        c = int(fc_c[r])
        cols = fi_c[r, :c].long()
        assert bool((cols[1:] > cols[:-1]).all()), r
        assert int(cols[-1]) < int(n[r]), r
        if plant is None:
            # the single-row indexer is the CUDA-core kernel: within its rounding of the tensor-core sum
            assert torch.allclose(fs_c[r, :c], sc[0, cols], rtol=0, atol=2e-3 * float(w[r].sum())), r

    if plant is not None:
        fails = _fused_fail_count(ops, dims, qI, kI, w, bias, scale, shift, q_pos0, chunk)
        assert fails > 0, plant


def test_fused_candidate_scores_are_the_materialised_scores(cuda_ok):
    """Bit for bit: the fused pass's candidate scores are the tensor-core scores the materialised pass
    writes (same kernel epilogue), here read from gsa_indexer_scores of the same chunk."""
    from gsa_b200 import ops

    dims = ops.make_dims(4096, 32, 8, 128, 8, 64)
    Lq = Lkv = 12000
    qI, kI, w, bias, shift = _inputs(1, Lq, Lkv, seed=3)
    scale = 1 / math.sqrt(64)
    fi, fs, fc, _ = ops.indexer_survivors(dims, qI, kI, w, bias, scale, shift, K_EFF, chunk_rows=Lq, fused=True)
    assert ops.last_survivor_path == "fused"
    rows = torch.arange(9000, 12000, 97)
    full = ops.indexer_scores(dims, qI[:, 9000:], kI, w.view(1, Lq, -1)[:, 9000:], bias, scale, q_pos0=9000,
                              causal=True)
    torch.cuda.synchronize()
    full = full.view(Lq - 9000, -1).cpu()
    fi_c, fs_c, fc_c = fi.cpu(), fs.cpu(), fc.cpu()
    for r in rows.tolist():
        c = int(fc_c[r])
        cols = fi_c[r, :c].long()
        assert torch.equal(fs_c[r, :c], full[r - 9000, cols]), r


def test_layer_forward_fused_equals_materialised(cuda_ok):
    """A bf16 layer forward (20,000 tokens: thresholded rows) with the fused survivor pass equals
    the forward with the materialised one, bit for bit."""
    from gsa_b200 import GatedSparseAttention, GSAConfig, ops

    cfg = GSAConfig(d_model=1024, n_heads=8, n_kv_heads=2, d_indexer=64, n_indexer_heads=8, k_base=2048,
                    k_min=256, k_max=4096, max_position_embeddings=32768)
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).to(DEV).to(torch.bfloat16).eval()
    x = torch.randn(1, 20000, 1024, generator=torch.Generator().manual_seed(1)).to(DEV, torch.bfloat16)
    cap_f, cap_m = {}, {}
    saved = ops.FUSED_SURVIVORS
    try:
        with torch.no_grad():
            ops.FUSED_SURVIVORS = True
            out_f = m._forward_impl(x, None, None, False, False, capture=cap_f)[0]
            assert ops.last_survivor_path == "fused"
            ops.FUSED_SURVIVORS = False
            out_m = m._forward_impl(x, None, None, False, False, capture=cap_m)[0]
            assert ops.last_survivor_path == "materialised"
    finally:
        ops.FUSED_SURVIVORS = saved
    torch.cuda.synchronize()
    assert torch.equal(cap_f["k_t"], cap_m["k_t"])
    assert torch.equal(cap_f["cnt"], cap_m["cnt"])
    valid = torch.arange(cap_m["sel"].shape[1], device=DEV).view(1, -1) < cap_m["cnt"].view(-1, 1).long()
    assert torch.equal(cap_f["sel"][valid], cap_m["sel"][valid])   # entries past a row's count are unset
    assert torch.equal(out_f, out_m)
