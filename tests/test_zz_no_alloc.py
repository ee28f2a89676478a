"""gsa_indexer_select_static (score scratch in a fixed library-owned buffer, no allocation)
returns what gsa_indexer_select (caller workspace) returns, on two calls in a row, both through
the C ABI.  Also: the second call changes the device's free memory by nothing, and the call
zeroes row_stats itself (the buffer is passed in dirty)."""

import ctypes as C
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(B, Lq, Lkv, HI, dI, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    qI = (torch.randn(B, Lq, HI * dI, generator=g) * 1.3).to(dtype)
    kI = (torch.randn(B, Lkv, dI, generator=g) * 1.4).to(dtype)
    w = torch.sigmoid(torch.randn(B * Lq, HI, generator=g) * 0.3)
    bias = torch.randn(HI, generator=g) * 0.1
    shift = 0.5 * w.sum(-1)
    return [t.to(DEV) for t in (qI, kI, w, bias, shift)]


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _run(lib, static, dims, dtype_code, B, Lq, Lkv, q_pos0, causal, qI, kI, w, bias, shift, k_eff,
         row_stats, workspace=None, chunk_rows=0, check_free=False):
    R = B * Lq
    cand_idx = torch.full((R, k_eff), -1, device=DEV, dtype=torch.int32)
    cand_score = torch.zeros(R, k_eff, device=DEV, dtype=torch.float32)
    cand_count = torch.full((R,), -1, device=DEV, dtype=torch.int32)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    common = (C.byref(dims), dtype_code, B, Lq, Lkv, q_pos0, int(causal), _p(qI), qI.stride(1), qI.stride(0),
              _p(kI), kI.stride(1), kI.stride(0), _p(w), _p(bias), 1.0 / math.sqrt(kI.shape[-1]), _p(shift),
              k_eff, _p(cand_idx), _p(cand_score), _p(cand_count), _p(row_stats))
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    if static:
        st = lib.gsa_indexer_select_static(*common, stream)
    else:
        st = lib.gsa_indexer_select(*common, chunk_rows, _p(workspace), workspace.numel(), stream)
    assert st == 0, st
    torch.cuda.synchronize()
    if check_free:
        assert torch.cuda.mem_get_info()[0] == free_before, "the call changed the free device memory"
    return cand_idx.cpu(), cand_score.cpu(), cand_count.cpu()


def _sorted_rows(idx, score, count):
    rows = []
    for r in range(idx.shape[0]):
        n = int(count[r])
        order = torch.argsort(idx[r, :n])
        rows.append((idx[r, :n][order], score[r, :n][order]))
    return rows


@pytest.mark.parametrize("dtype,B,Lq,Lkv,HI,q_pos0,causal,k_eff", [
    (torch.bfloat16, 2, 1200, 1200, 8, 0, True, 256),       # tensor-core indexer, one chunk
    (torch.bfloat16, 1, 1000, 40000, 8, 39000, True, 512),  # 419-row chunks: three of them
    (torch.float32, 1, 300, 500, 4, 200, True, 64),          # fp32 indexer kernel
])
def test_static_scratch_select_matches_workspace_select(cuda_ok, dtype, B, Lq, Lkv, HI, q_pos0, causal, k_eff):
    from gsa_b200 import _lib, ops

    lib = _lib.lib()
    dI = 64
    dims = ops.make_dims(4096, 32, 8, 128, HI, dI)
    code = ops.dtype_code(dtype)
    qI, kI, w, bias, shift = _inputs(B, Lq, Lkv, HI, dI, dtype, seed=7)
    R = B * Lq

    # the existing entry point with a caller workspace (chunks of 128 rows)
    chunk = 128
    ws = torch.empty(lib.gsa_workspace_size(chunk, Lkv), device=DEV, dtype=torch.uint8)
    ref_stats = torch.zeros(R, 3, device=DEV, dtype=torch.float64)
    ref = _run(lib, False, dims, code, B, Lq, Lkv, q_pos0, causal, qI, kI, w, bias, shift, k_eff, ref_stats,
               workspace=ws, chunk_rows=chunk)
    ref_rows = _sorted_rows(*ref)

    stats = torch.full((R, 3), 123.0, device=DEV, dtype=torch.float64)  # dirty: the call zeroes it
    for call in range(2):
        # the first call on the device may do its one-time set-up; the second must allocate nothing
        out = _run(lib, True, dims, code, B, Lq, Lkv, q_pos0, causal, qI, kI, w, bias, shift, k_eff, stats,
                   check_free=call == 1)
        assert torch.equal(out[2], ref[2]), f"call {call}: candidate counts differ"
        for r, ((i0, s0), (i1, s1)) in enumerate(zip(ref_rows, _sorted_rows(*out))):
            assert torch.equal(i0, i1), f"call {call}: row {r} candidates differ"
            assert torch.equal(s0, s1), f"call {call}: row {r} candidate scores differ"
        # fp64 sums accumulated by atomics in a different order: equal to rounding
        assert torch.equal(stats[:, 2].cpu(), ref_stats[:, 2].cpu())
        assert torch.allclose(stats[:, :2].cpu(), ref_stats[:, :2].cpu(), rtol=1e-9, atol=1e-9)
    ops.check_device_error()


def test_static_scratch_rejects_key_length_beyond_its_buffer(cuda_ok):
    from gsa_b200 import _lib, ops

    lib = _lib.lib()
    dims = ops.make_dims(4096, 32, 8, 128, 8, 64)
    too_long = (64 << 20) // 4 + 1
    p = C.c_void_p(256)  # stand-in pointers: the size check returns before any is used
    st = lib.gsa_indexer_select_static(C.byref(dims), 1, 1, 1, too_long, 0, 1, p, 512, 0, p, 64, 0,
                                       p, p, 0.125, p, 16, p, p, p, None, None)
    assert st == 3  # GSA_ERR_WORKSPACE
