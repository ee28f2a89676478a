"""Final selection (gsa_select_finalize): the warp-per-row kernel (no mask asked) and the per-row
CTA kernel (mask asked) keep the same k_t candidates of every row -- the k_t largest scores,
ties lower column first, in ascending column order -- and both equal the oracle's stable top-k.
Rows: random scores, heavy ties at a few levels (the radix branch of the warp kernel), all
equal, negative scores, ulp-level steps, k_t = 0, k_t >= candidates, empty rows."""

import numpy as np
import pytest
import torch

import gsa_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_warp_and_block_selection_agree_with_oracle(cuda_ok):
    from gsa_b200 import ops

    g = torch.Generator().manual_seed(11)
    R, ld = 64, 6000
    cols = torch.sort(torch.randperm(20000, generator=g)[:ld]).values.int().repeat(R, 1)
    scores = torch.rand(R, ld, generator=g) * 3
    scores[1] = 0.75                                          # all equal
    scores[2] = torch.round(scores[2] * 4) / 4                # 13 levels: boundary bins of ~460
    scores[3] = -scores[3]                                    # negative
    scores[4, ::2] = scores[4, 1::2]                          # pairs of equal scores
    scores[5] = 1.0 + torch.arange(ld).float() * 1e-7         # a narrow range, ulp-level steps
    count = torch.full((R,), ld, dtype=torch.int32)
    count[6] = 3000
    count[7] = 0
    k = torch.randint(1, ld, (R,), generator=g).int()
    k[8] = 0
    k[9] = ld + 5
    k[10] = 2999
    k[6] = 2500
    k[[1, 2, 5]] = torch.tensor([1234, 2500, 4000], dtype=torch.int32)
    args = (cols.to(DEV), scores.to(DEV), count.to(DEV), k.to(DEV))
    sel_w, cnt_w, _ = ops.select_finalize(*args, want_mask=False, sel_ld=ld)
    sel_b, cnt_b, mask_b = ops.select_finalize(*args, want_mask=True, sel_ld=ld)
    torch.cuda.synchronize()
    ops.check_device_error()
    assert torch.equal(cnt_w, cnt_b)
    for r in range(R):
        n = int(cnt_w[r])
        assert torch.equal(sel_w[r, :n], sel_b[r, :n]), r
        m = int(count[r])
        kk = min(max(int(k[r]), 0), m)
        assert n == kk, r
        if m == 0:
            continue
        ref_pos = O.topk_sets_stable(scores[r:r + 1, :m], torch.tensor([kk]))[0]
        ref = np.sort(cols[r, ref_pos].numpy())
        assert np.array_equal(sel_w[r, :n].cpu().numpy(), ref), r
