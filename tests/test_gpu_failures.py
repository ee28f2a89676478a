"""Device-side failure handling, exercised without a GPU fault.

Every kernel records failures in a device error word instead of trapping; the host reads (and
clears) it with gsa_get_device_error.  Two routes into it:

* an out-of-range key index in a row's selection: the sparse SDPA checks each index before the
  access, records GSA_ERR_INDEX and reads a zero row in its place, so the output stays finite;
* a bounded mbarrier wait that runs out: the diagnostic entry point waits on a barrier nothing
  arrives on, with a short poll limit; it records GSA_ERR_TIMEOUT and returns, and the context
  stays usable for the next launch.

The reference has no device code; its only failure handling is a try/except around its Triton
calls (gsa/kernels/triton_sparse_attn.py:196-212)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
GSA_ERR_TIMEOUT, GSA_ERR_INDEX = 4, 6


def _sdpa_case(dtype, B=1, Lq=4, Lkv=100, H=8, Hk=2, D=64, k=16, seed=3):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Lq, H, D, generator=g).to(DEV, dtype)
    kv = torch.randn(B, Lkv, 2, Hk, D, generator=g).to(DEV, dtype)
    sel = torch.stack([torch.randperm(Lkv, generator=g)[:k] for _ in range(B * Lq)]).int().to(DEV)
    cnt = torch.full((B * Lq,), k, dtype=torch.int32, device=DEV)
    return q, kv, sel, cnt


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_out_of_range_selection_index_is_reported_and_read_as_zero(cuda_ok, dtype):
    from gsa_b200 import ops

    dims = ops.make_dims(512, 8, 2, 64, 4, 32)
    q, kv, sel, cnt = _sdpa_case(dtype)
    ops.check_device_error()                      # start from a clear error word
    good = ops.sparse_sdpa(dims, q, kv[:, :, 0], kv[:, :, 1], sel, cnt, None, 0.125)
    torch.cuda.synchronize()
    ops.check_device_error()
    bad = sel.clone()
    bad[1, 3] = 100                               # == Lkv: one past the last key
    bad[2, 0] = -7
    out = ops.sparse_sdpa(dims, q, kv[:, :, 0], kv[:, :, 1], bad, cnt, None, 0.125)
    torch.cuda.synchronize()
    from gsa_b200 import _lib
    import ctypes as C
    code = C.c_int(0)
    _lib.call("gsa_get_device_error", C.byref(code), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code.value == GSA_ERR_INDEX
    assert bool(torch.isfinite(out.float()).all())
    # the rows without a bad index are unaffected; the read cleared the word
    assert torch.equal(out[0, 0], good[0, 0]) and torch.equal(out[0, 3], good[0, 3])
    ops.check_device_error()


def test_bounded_wait_runs_out_and_reports_a_timeout(cuda_ok):
    from gsa_b200 import ops

    ops.check_device_error()
    assert ops.selftest_bounded_wait(4096) == GSA_ERR_TIMEOUT
    # the read cleared the word and the context still runs kernels
    ops.check_device_error()
    dims = ops.make_dims(512, 8, 2, 64, 4, 32)
    q, kv, sel, cnt = _sdpa_case(torch.bfloat16)
    out = ops.sparse_sdpa(dims, q, kv[:, :, 0], kv[:, :, 1], sel, cnt, None, 0.125)
    torch.cuda.synchronize()
    ops.check_device_error()
    kk = kv[0, sel[1].long(), 0].float().repeat_interleave(4, dim=1)
    vv = kv[0, sel[1].long(), 1].float().repeat_interleave(4, dim=1)
    p = torch.softmax(torch.einsum("hd,chd->hc", q[0, 1].float(), kk) * 0.125, dim=-1)
    ref = torch.einsum("hc,chd->hd", p, vv)
    assert float((out[0, 1].float() - ref).norm() / ref.norm()) < 2e-2

