"""Tensor-level wrappers over the C ABI (include/gsa_b200.h).

Each function checks devices, dtypes and layouts, allocates its outputs with torch (the ABI
itself allocates nothing), and calls one entry point on the current CUDA stream.  Nothing here
computes on the CPU: a tensor that is not on a CUDA device is an error.
"""

from __future__ import annotations

import ctypes as C
import os

import torch

from . import _lib
from ._lib import ACT, DTYPE_BF16, DTYPE_F32, Dims, ProjLayout, TopkParams

DEBUG = os.environ.get("GSA_DEBUG", "0") == "1"
# number of (indexer, top-k) chunk launches of the last indexer_select call
last_chunk_count = 0
last_survivor_path = None  # "fused" or "materialised": the survivor pass the last call took
# bound of the chunk score scratch of the layer's indexer pass (fewer, larger chunks amortise
# each launch's tail; the scratch lives only during the call)
SCORE_CHUNK_BYTES = 4 << 30


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return DTYPE_F32
    if dt == torch.bfloat16:
        return DTYPE_BF16
    raise NotImplementedError(f"GSA B200 kernels support float32 and bfloat16, got {dt}")


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("GSA B200 ops take CUDA tensors only (there is no CPU path)")


def check_device_error():
    """Raise if a kernel recorded a device-side error (bounded wait timeout, bad index)."""
    code = C.c_int(0)
    _lib.call("gsa_get_device_error", C.byref(code), _stream())
    if code.value:
        raise _lib.GSAError("device", code.value)


def _after(name):
    if DEBUG:
        torch.cuda.synchronize()
        check_device_error()


def make_dims(d_model, n_heads, n_kv_heads, d_head, n_idx_heads, d_idx, gate_act="sigmoid",
              idx_act="sigmoid") -> Dims:
    return Dims(d_model, n_heads, n_kv_heads, d_head, n_idx_heads, d_idx, ACT[gate_act], ACT[idx_act])


def proj_epilogue(dims: Dims, layout: ProjLayout, proj: torch.Tensor, positions: torch.Tensor,
                  cos_tab: torch.Tensor, sin_tab: torch.Tensor, has_g1: bool, return_kv: bool = False,
                  kv_out: torch.Tensor | None = None, ki_out: torch.Tensor | None = None):
    """q, k (RoPE), v (G2), g1 gate, indexer head weights w and row shift from the fused
    projection output ``proj`` [T, Ncat].  k and v are views of one interleaved [T, 2, Hk, D]
    buffer; with ``return_kv`` that buffer is returned in their place: (q, kv, g1, w, shift).

    ``kv_out`` [B, L, 2, Hk, D] (T = B*L; a view into a KV cache with a larger batch stride) and
    ``ki_out`` [B, L, d_I] receive K/V and the indexer keys directly; kv_out is then the returned kv."""
    _cuda(proj, positions, cos_tab, sin_tab)
    T = proj.shape[0]
    H, Hk, D, HI = dims.n_heads, dims.n_kv_heads, dims.d_head, dims.n_idx_heads
    dt = proj.dtype
    q = torch.empty(T, H, D, device=proj.device, dtype=dt)
    g1 = torch.empty(T, H, D, device=proj.device, dtype=dt) if has_g1 else None
    w = torch.empty(T, HI, device=proj.device, dtype=torch.float32)
    shift = torch.empty(T, device=proj.device, dtype=torch.float32)
    pos = positions.reshape(-1).to(torch.int64).contiguous()
    assert proj.stride(1) == 1 and pos.numel() == T
    cos_tab = cos_tab.contiguous()
    sin_tab = sin_tab.contiguous()
    if kv_out is None:
        # K and V interleaved per token ([T, 2, Hk, D]): the sparse SDPA moves a key as one copy
        kv = torch.empty(T, 2, Hk, D, device=proj.device, dtype=dt)
        k, v = kv[:, 0], kv[:, 1]
        _lib.call("gsa_proj_epilogue", C.byref(dims), C.byref(layout), dtype_code(dt), T, _p(proj),
                  proj.stride(0), _p(pos), _p(cos_tab), _p(sin_tab), dtype_code(cos_tab.dtype),
                  cos_tab.shape[0], _p(q), _p(k), _p(v), kv.stride(0), _p(g1), _p(w), _p(shift), _stream())
    else:
        _cuda(kv_out, ki_out)
        B, L = kv_out.shape[0], kv_out.shape[1]
        assert B * L == T and kv_out.dtype == dt and tuple(kv_out.shape[2:]) == (2, Hk, D)
        assert kv_out.stride(4) == 1 and kv_out.stride(3) == D and kv_out.stride(2) == Hk * D
        kv = kv_out
        k, v = kv[:, :, 0], kv[:, :, 1]
        ki_ld = ki_bs = 0
        if ki_out is not None:
            assert ki_out.shape == (B, L, dims.d_idx) and ki_out.stride(2) == 1 and ki_out.dtype == dt
            ki_ld, ki_bs = ki_out.stride(1), ki_out.stride(0)
        _lib.call("gsa_proj_epilogue_cache", C.byref(dims), C.byref(layout), dtype_code(dt), B, L, _p(proj),
                  proj.stride(0), _p(pos), _p(cos_tab), _p(sin_tab), dtype_code(cos_tab.dtype),
                  cos_tab.shape[0], _p(q), _p(k), _p(v), kv.stride(1), kv.stride(0), _p(ki_out), ki_ld, ki_bs,
                  _p(g1), _p(w), _p(shift), _stream())
    _after("proj_epilogue")
    if return_kv:
        return q, kv, g1, w, shift
    return q, k, v, g1, w, shift


def proj_fused_rows(dims: Dims) -> int:
    return int(_lib.lib().gsa_proj_fused_rows(C.byref(dims)))


def proj_fused(dims: Dims, wp: torch.Tensor, bias: torch.Tensor, x2d: torch.Tensor, B: int, L: int,
               positions: torch.Tensor, cos_tab: torch.Tensor, sin_tab: torch.Tensor,
               kv_out: torch.Tensor | None = None, ki_out: torch.Tensor | None = None):
    """The fused projection GEMM (gsa_proj_fused) on x2d [B*L, d_model] bf16: (q [T, H, D], kv
    [B, L, 2, Hk, D] (or ``kv_out``, a KV-cache view), g1 [T, H, D], w [T, H_I] fp32, shift [T] fp32,
    qI [B, L, H_I*d_I], kI [B, L, d_I] (or ``ki_out``)).  None when the kernel does not take these
    shapes (the caller then runs the GEMM and gsa_proj_epilogue)."""
    _cuda(wp, bias, x2d, positions, cos_tab, sin_tab, kv_out, ki_out)
    T = x2d.shape[0]
    H, Hk, D, HI, dI = dims.n_heads, dims.n_kv_heads, dims.d_head, dims.n_idx_heads, dims.d_idx
    dev, dt = x2d.device, x2d.dtype
    if dt != torch.bfloat16 or x2d.stride(1) != 1 or wp.dtype != dt or not wp.is_contiguous():
        return None
    q = torch.empty(T, H, D, device=dev, dtype=dt)
    g1 = torch.empty(T, H, D, device=dev, dtype=dt)
    w = torch.empty(T, HI, device=dev, dtype=torch.float32)
    shift = torch.empty(T, device=dev, dtype=torch.float32)
    qI = torch.empty(B, L, HI * dI, device=dev, dtype=dt)
    kv = kv_out if kv_out is not None else torch.empty(B, L, 2, Hk, D, device=dev, dtype=dt)
    kI = ki_out if ki_out is not None else torch.empty(B, L, dI, device=dev, dtype=dt)
    k, v = kv[:, :, 0], kv[:, :, 1]
    pos = positions.reshape(-1).to(torch.int64).contiguous()
    cos_tab, sin_tab = cos_tab.contiguous(), sin_tab.contiguous()
    st = _lib.lib().gsa_proj_fused(C.byref(dims), dtype_code(dt), T, L, _p(x2d), x2d.stride(0), _p(wp),
                                   _p(bias.float().contiguous()), _p(pos), 0, _p(cos_tab), _p(sin_tab),
                                   dtype_code(cos_tab.dtype), cos_tab.shape[0], _p(q), _p(k), _p(v), kv.stride(1),
                                   kv.stride(0), _p(g1), _p(qI), qI.stride(1), _p(kI), kI.stride(1), kI.stride(0),
                                   _p(w), _p(shift), _stream())
    if st == 2:  # GSA_ERR_UNSUPPORTED
        return None
    if st != 0:
        raise _lib.GSAError("gsa_proj_fused", st)
    _after("proj_fused")
    return q, kv, g1, w, shift, qI, kI


def indexer_scores(dims: Dims, qI: torch.Tensor, kI: torch.Tensor, w: torch.Tensor,
                   bias: torch.Tensor, scale: float, q_pos0: int = 0, causal: bool = True,
                   shift=None, row_stats=None) -> torch.Tensor:
    """Materialised indexer scores [B, Lq, Lkv] fp32 with -inf at causally masked entries.
    qI [B, Lq, H_I*d_I] and kI [B, Lkv, d_I] may be row-strided views (last dim contiguous)."""
    _cuda(qI, kI, w, bias)
    B, Lq, _ = qI.shape
    Lkv = kI.shape[1]
    assert qI.stride(2) == 1 and kI.stride(2) == 1 and qI.dtype == kI.dtype
    ld = (Lkv + 3) // 4 * 4
    # masked entries keep the -inf fill, so the kernels need not write them
    scores = torch.full((B * Lq, ld), float("-inf"), device=qI.device, dtype=torch.float32)
    w = w.reshape(B * Lq, -1).float().contiguous()
    bias = bias.float().contiguous()
    _lib.call("gsa_indexer_scores", C.byref(dims), dtype_code(qI.dtype), B, Lq, Lkv, q_pos0,
              int(causal), 0, _p(qI), qI.stride(1), qI.stride(0), _p(kI),
              kI.stride(1), kI.stride(0), _p(w), _p(bias), float(scale), _p(shift), _p(scores), ld,
              _p(row_stats), _stream())
    _after("indexer_scores")
    return scores[:, :Lkv].reshape(B, Lq, Lkv)


def row_stats(scores2d: torch.Tensor) -> torch.Tensor:
    """fp64 [R, 3] = (sum, sum of squares, finite count) per row of a fp32 [R, n] matrix."""
    _cuda(scores2d)
    s = scores2d.float()
    if s.stride(1) != 1:
        s = s.contiguous()
    R, n = s.shape
    stats = torch.zeros(R, 3, device=s.device, dtype=torch.float64)
    _lib.call("gsa_row_stats", R, n, _p(s), s.stride(0), _p(stats), _stream())
    _after("row_stats")
    return stats


def row_summary(scores2d: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """fp32 [R, 5] = (valid count, mean, std, max of the masked scores, softmax entropy) per row of
    a score matrix holding values of ``dtype`` (the statistics of the entropy and learned
    adaptive-k methods, adaptive_topk.py:84-127, rounded to ``dtype``)."""
    _cuda(scores2d)
    s = scores2d.float()
    if s.stride(1) != 1:
        s = s.contiguous()
    R, n = s.shape
    out = torch.empty(R, 5, device=s.device, dtype=torch.float32)
    _lib.call("gsa_row_summary", R, n, _p(s), s.stride(0), dtype_code(dtype), _p(out), _stream())
    _after("row_summary")
    return out


def topk_candidates(scores2d: torch.Tensor, k_eff: int, Lq: int | None = None, q_pos0: int = 0,
                    causal: bool = False, row_center: torch.Tensor | None = None,
                    row_stats: torch.Tensor | None = None):
    """k_eff largest finite scores per row, ascending column order (int32 idx, fp32 score,
    int32 count).  Unfilled slots hold column 0.  ``row_center`` [R]: every finite score of row
    r lies in [0, 2 row_center[r]] (enables the two-pass bounded-range selection)."""
    _cuda(scores2d)
    s = scores2d if scores2d.dtype == torch.float32 else scores2d.float()
    if s.stride(1) != 1:
        s = s.contiguous()
    R, n = s.shape
    idx = torch.zeros(R, k_eff, device=s.device, dtype=torch.int32)
    sc = torch.zeros(R, k_eff, device=s.device, dtype=torch.float32)
    cnt = torch.empty(R, device=s.device, dtype=torch.int32)
    if row_center is not None:
        row_center = row_center.float().contiguous()
    _lib.call("gsa_topk_candidates", R, Lq or R, n, q_pos0, int(causal), _p(s), s.stride(0),
              _p(row_center), _p(row_stats), int(k_eff), _p(idx), _p(sc), _p(cnt), _stream())
    _after("topk_candidates")
    return idx, sc, cnt


def row_variance(stats: torch.Tensor, n_cols: int, dt: torch.dtype, shift=None):
    R = stats.shape[0]
    var = torch.empty(R, device=stats.device, dtype=torch.float32)
    total = torch.empty(2, device=stats.device, dtype=torch.float64)
    _lib.call("gsa_row_variance", R, n_cols, dtype_code(dt), _p(stats), _p(shift), _p(var),
              _p(total), _stream())
    _after("row_variance")
    return var, total


def adaptive_k(stats, var, total, n_cols: int, dt: torch.dtype, k_base: int, k_min: int,
               k_max: int, use_adaptive: bool, temperature: float) -> torch.Tensor:
    R = stats.shape[0]
    k = torch.empty(R, device=stats.device, dtype=torch.int32)
    p = TopkParams(k_base, k_min, k_max, int(use_adaptive), float(temperature))
    _lib.call("gsa_adaptive_k", R, n_cols, dtype_code(dt), C.byref(p), _p(var), _p(total),
              _p(stats), _p(k), _stream())
    _after("adaptive_k")
    return k


def decode_workspace_bytes(dims: Dims, tp: TopkParams, dt: torch.dtype, B: int, L: int, n_keys: int) -> int:
    return int(_lib.lib().gsa_decode_workspace_size(C.byref(dims), C.byref(tp), dtype_code(dt), B, L, n_keys))


DECODE_ALL, DECODE_SCORE, DECODE_ATTEND = 0, 1, 2


def decode_attend(dims: Dims, layout: ProjLayout, tp: TopkParams, proj: torch.Tensor, B: int, L: int, past: int,
                  positions, cos_tab, sin_tab, kv_store: torch.Tensor, ki_store: torch.Tensor, idx_bias: torch.Tensor,
                  idx_scale: float, attn_scale: float, workspace: torch.Tensor, allreduce=None) -> torch.Tensor:
    """The attention of one step between its two GEMMs in native calls (gsa_decode_attend):
    the new tokens' K, V, k^I appended to the stores at slot ``past``, the indexer over all
    past + L keys, the selection and the gated SDPA.  ``allreduce(t)`` (sequences spread over
    several GPUs): the step runs in two phases with the variance sum all-reduced in between.
    Returns attn [B*L, H*D]."""
    dt = proj.dtype
    attn = torch.empty(B * L, dims.n_heads * dims.d_head, device=proj.device, dtype=dt)
    if positions is not None:
        positions = positions.reshape(-1).to(torch.int64).contiguous()
    args = [C.byref(dims), C.byref(layout), C.byref(tp), dtype_code(dt), B, L, past, _p(proj), proj.stride(0),
            _p(positions), _p(cos_tab), _p(sin_tab), dtype_code(cos_tab.dtype), cos_tab.shape[0], _p(kv_store),
            kv_store.stride(0), _p(ki_store), ki_store.stride(0), _p(idx_bias), float(idx_scale), float(attn_scale),
            _p(attn), None]
    tail = [_p(workspace), workspace.numel(), _stream()]
    if allreduce is None:
        _lib.call("gsa_decode_attend", *args, None, DECODE_ALL, *tail)
    else:
        total = torch.empty(2, device=proj.device, dtype=torch.float64)
        _lib.call("gsa_decode_attend", *args, _p(total), DECODE_SCORE, *tail)
        total = allreduce(total)
        _lib.call("gsa_decode_attend", *args, _p(total), DECODE_ATTEND, *tail)
    _after("decode_attend")
    return attn


def select_finalize(cand_idx, cand_score, cand_count, k, want_mask: bool = False, sel_ld: int | None = None):
    """The k[r] best candidates of each row, ascending column order: (sel [R, sel_ld], count [R],
    mask [R, cand_ld] or None).  sel_ld defaults to the candidate row length."""
    R, k_eff = cand_idx.shape
    sel = torch.empty(R, sel_ld or k_eff, device=cand_idx.device, dtype=torch.int32)
    cnt = torch.empty(R, device=cand_idx.device, dtype=torch.int32)
    mask = torch.empty(R, k_eff, device=cand_idx.device, dtype=torch.uint8) if want_mask else None
    _lib.call("gsa_select_finalize", R, k_eff, _p(cand_idx), _p(cand_score), _p(cand_count), _p(k),
              _p(sel), sel.stride(0), _p(cnt), _p(mask), _stream())
    _after("select_finalize")
    return sel, cnt, mask


def _kv_rows(t: torch.Tensor) -> torch.Tensor:
    """[B, Lkv, Hk, D] with unit-stride rows of Hk*D elements and a batch stride that holds the
    Lkv key rows (a KV cache may hold room for more)."""
    B, L, Hk, D = t.shape
    if t.stride(3) != 1 or t.stride(2) != D or (B > 1 and (t.stride(0) < L * t.stride(1) or t.stride(0) % 8)):
        t = t.contiguous()
    return t


def _kv_bstride(t: torch.Tensor) -> int:
    return t.stride(0) if t.shape[0] > 1 else t.shape[1] * t.stride(1)


def sparse_sdpa(dims: Dims, q, k, v, sel_idx, sel_count, gate, scale: float) -> torch.Tensor:
    """q [B, Lq, H, D]; k, v [B, Lkv, Hk, D] (separate, or views of one interleaved
    [B, Lkv, 2, Hk, D] buffer); sel [B*Lq, ld] int32; gate like q or None."""
    _cuda(q, k, v, sel_idx, sel_count, gate)
    B, Lq = q.shape[0], q.shape[1]
    Lkv = k.shape[1]
    q = q.contiguous()
    k = _kv_rows(k)
    v = _kv_rows(v)
    if k.stride(1) != v.stride(1) or _kv_bstride(k) != _kv_bstride(v):
        k, v = k.contiguous(), v.contiguous()
    gate = gate.contiguous() if gate is not None else None
    out = torch.empty_like(q)
    # few rows (decode): room for per-key-range partials, so that every CTA streams keys
    ws_bytes = int(_lib.lib().gsa_sdpa_workspace_size(C.byref(dims), B, Lq)) if q.dtype == torch.bfloat16 else 0
    ws = torch.empty(ws_bytes, device=q.device, dtype=torch.uint8) if ws_bytes else None
    _lib.call("gsa_sparse_sdpa_strided", C.byref(dims), dtype_code(q.dtype), B, Lq, Lkv, _p(q), _p(k), _p(v),
              k.stride(1), _kv_bstride(k), _p(sel_idx), sel_idx.stride(0), _p(sel_count), _p(gate), _p(out),
              float(scale), _p(ws), ws_bytes, _stream())
    _after("sparse_sdpa")
    return out


def sparse_sdpa_lse(dims: Dims, q, k, v, sel_idx, sel_count, scale: float):
    """Ungated sparse SDPA that also returns the per-(row, head) natural-log sum-exp of the scaled
    scores [B*Lq, H] fp32 (the backward's softmax statistics)."""
    _cuda(q, k, v, sel_idx, sel_count)
    B, Lq = q.shape[0], q.shape[1]
    Lkv = k.shape[1]
    q = q.contiguous()
    k = _kv_rows(k)
    v = _kv_rows(v)
    if k.stride(1) != v.stride(1) or _kv_bstride(k) != _kv_bstride(v):
        k, v = k.contiguous(), v.contiguous()
    out = torch.empty_like(q)
    lse = torch.empty(B * Lq, dims.n_heads, device=q.device, dtype=torch.float32)
    _lib.call("gsa_sparse_sdpa_lse", C.byref(dims), dtype_code(q.dtype), B, Lq, Lkv, _p(q), _p(k), _p(v),
              k.stride(1), _kv_bstride(k), _p(sel_idx), sel_idx.stride(0), _p(sel_count), None, _p(out), _p(lse),
              float(scale), _stream())
    _after("sparse_sdpa_lse")
    return out, lse


def sparse_sdpa_probs(dims: Dims, q, k, idx, mask, lse, scale: float) -> torch.Tensor:
    """Attention probabilities [B, Lq, H, k_eff] (dtype of q) of the candidates ``idx``
    [B*Lq, k_eff] that ``mask`` (uint8, or None: all) keeps, from the per-(row, head) log-sum-exp
    ``lse`` [B*Lq, H] of the SDPA over the same keys; 0 for candidates not kept."""
    _cuda(q, k, idx, mask, lse)
    B, Lq, H, D = q.shape
    Lkv = k.shape[1]
    q = q.contiguous()
    k = _kv_rows(k)
    idx = idx.to(torch.int32).contiguous()
    mask = mask.to(torch.uint8).contiguous() if mask is not None else None
    R, k_eff = idx.shape
    out = torch.empty(R, H, k_eff, device=q.device, dtype=q.dtype)
    _lib.call("gsa_sparse_sdpa_probs", C.byref(dims), dtype_code(q.dtype), B, Lq, Lkv, _p(q), _p(k), k.stride(1),
              _kv_bstride(k), _p(idx), _p(mask), k_eff, k_eff, _p(lse.contiguous()), float(scale), _p(out), _stream())
    _after("sparse_sdpa_probs")
    return out.view(B, Lq, H, k_eff)


def sparse_sdpa_lse_gated(dims: Dims, q, k, v, sel_idx, sel_count, gate, scale: float):
    """sparse_sdpa with the G1 gate in its epilogue that also returns the log-sum-exp [B*Lq, H]."""
    _cuda(q, k, v, sel_idx, sel_count, gate)
    B, Lq = q.shape[0], q.shape[1]
    Lkv = k.shape[1]
    q = q.contiguous()
    k = _kv_rows(k)
    v = _kv_rows(v)
    if k.stride(1) != v.stride(1) or _kv_bstride(k) != _kv_bstride(v):
        k, v = k.contiguous(), v.contiguous()
    gate = gate.contiguous() if gate is not None else None
    out = torch.empty_like(q)
    lse = torch.empty(B * Lq, dims.n_heads, device=q.device, dtype=torch.float32)
    _lib.call("gsa_sparse_sdpa_lse", C.byref(dims), dtype_code(q.dtype), B, Lq, Lkv, _p(q), _p(k), _p(v),
              k.stride(1), _kv_bstride(k), _p(sel_idx), sel_idx.stride(0), _p(sel_count), _p(gate), _p(out),
              _p(lse), float(scale), _stream())
    _after("sparse_sdpa_lse")
    return out, lse


def selftest_bounded_wait(wait_limit: int = 4096) -> int:
    """Run the bounded-wait diagnostic kernel and return the device error code it left (expected:
    GSA_ERR_TIMEOUT, 4); the error word is cleared by the read."""
    _lib.call("gsa_selftest_bounded_wait", int(wait_limit), _stream())
    code = C.c_int(0)
    _lib.call("gsa_get_device_error", C.byref(code), _stream())
    return code.value


def sparse_sdpa_backward(dims: Dims, q, k, v, sel_idx, sel_count, o, d_o, lse, scale: float):
    """Gradients of the ungated sparse SDPA: (dq [B, Lq, H, D], dk, dv [B, Lkv, Hk, D]), fp32."""
    _cuda(q, k, v, sel_idx, sel_count, o, d_o, lse)
    B, Lq, H, D = q.shape
    Lkv, Hk = k.shape[1], k.shape[2]
    q, o, d_o = q.contiguous(), o.contiguous(), d_o.contiguous().to(q.dtype)
    k = _kv_rows(k)
    v = _kv_rows(v)
    if k.stride(1) != v.stride(1) or _kv_bstride(k) != _kv_bstride(v):
        k, v = k.contiguous(), v.contiguous()
    dq = torch.empty(B, Lq, H, D, device=q.device, dtype=torch.float32)
    dkv = torch.zeros(B, Lkv, 2, Hk, D, device=q.device, dtype=torch.float32)
    dk, dv = dkv[:, :, 0], dkv[:, :, 1]
    _lib.call("gsa_sparse_sdpa_backward", C.byref(dims), dtype_code(q.dtype), B, Lq, Lkv, _p(q), _p(k), _p(v),
              k.stride(1), _kv_bstride(k), _p(sel_idx), sel_idx.stride(0), _p(sel_count), _p(o), _p(d_o),
              _p(lse.contiguous()), _p(dq), _p(dk), _p(dv), dk.stride(1), dk.stride(0), float(scale), _stream())
    _after("sparse_sdpa_backward")
    return dq, dk, dv


def add_rmsnorm(x: torch.Tensor, a, weight, eps: float, want_sum: bool = True, want_norm: bool = True):
    """(h = x + a, RMSNorm(h) * weight) over the last dimension (a None: no add, h = x).  Either
    output may be skipped; returns (h or None, y or None)."""
    _cuda(x, a, weight)
    d = x.shape[-1]
    x2 = x.reshape(-1, d)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    a2 = None
    if a is not None:
        a2 = a.reshape(-1, d)
        if a2.stride(1) != 1:
            a2 = a2.contiguous()
    T = x2.shape[0]
    h = torch.empty_like(x2) if (a is not None and want_sum) else None
    y = torch.empty_like(x2) if want_norm else None
    w = weight.contiguous() if weight is not None else None
    _lib.call("gsa_add_rmsnorm", dtype_code(x.dtype), T, d, _p(x2), x2.stride(0), _p(a2),
              a2.stride(0) if a2 is not None else 0, _p(w), float(eps), _p(h), d, _p(y), d, _stream())
    _after("add_rmsnorm")
    return (h.view(x.shape) if h is not None else None), (y.view(x.shape) if y is not None else None)


def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    """silu(gu[..., :n]) * gu[..., n:] for gu [..., 2n]."""
    _cuda(gu)
    n2 = gu.shape[-1]
    g2 = gu.reshape(-1, n2)
    if g2.stride(1) != 1:
        g2 = g2.contiguous()
    n = n2 // 2
    z = torch.empty(g2.shape[0], n, device=gu.device, dtype=gu.dtype)
    _lib.call("gsa_silu_mul", dtype_code(gu.dtype), g2.shape[0], n, _p(g2), g2.stride(0), _p(z), n, _stream())
    _after("silu_mul")
    return z.view(*gu.shape[:-1], n)


def apply_gate(x: torch.Tensor, logits: torch.Tensor, act: str, want_gate: bool = False):
    _cuda(x, logits)
    x = x.contiguous()
    logits = logits.contiguous()
    assert x.shape == logits.shape and x.dtype == logits.dtype
    out = torch.empty_like(x)
    gate = torch.empty_like(x) if want_gate else None
    _lib.call("gsa_apply_gate", dtype_code(x.dtype), ACT[act], x.numel(), _p(x), _p(logits), _p(out),
              _p(gate), _stream())
    _after("apply_gate")
    return out, gate


def _chunking(B: int, Lq: int, Lkv: int, chunk_rows: int | None):
    """(rows per indexer chunk, number of chunks).  Chunks hold whole sequences when a sequence's
    rows fit (so the short rows of many sequences share a launch), else rows of one sequence."""
    if chunk_rows is None:
        cap = max(1, SCORE_CHUNK_BYTES // (4 * ((Lkv + 3) // 4 * 4)))
        chunk_rows = min(B, cap // Lq) * Lq if cap >= Lq else cap
    if chunk_rows >= Lq:
        per = chunk_rows // Lq
        return chunk_rows, (B + per - 1) // per
    return chunk_rows, B * ((Lq + chunk_rows - 1) // chunk_rows)


def workspace_bytes(chunk_rows: int, n_cols: int) -> int:
    return int(_lib.lib().gsa_workspace_size(chunk_rows, n_cols))


def indexer_select(dims: Dims, qI, kI, w, bias, scale: float, shift, k_eff: int, q_pos0: int = 0,
                   causal: bool = True, chunk_rows: int | None = None, row_stats=None,
                   workspace=None, out=None):
    """Indexer + top-k candidates for all rows, chunk by chunk (no [Lq, Lkv] score matrix).

    qI [B, Lq, H_I*d_I], kI [B, Lkv, d_I] (row-strided views allowed).  Returns
    (cand_idx, cand_score, cand_count, row_stats) with rows = B*Lq; ``out`` may supply the first
    three (row-contiguous) to be filled in place."""
    _cuda(qI, kI, w, bias)
    B, Lq, _ = qI.shape
    Lkv = kI.shape[1]
    R = B * Lq
    dev = qI.device
    global last_chunk_count
    chunk_rows, last_chunk_count = _chunking(B, Lq, Lkv, chunk_rows)
    need = workspace_bytes(chunk_rows, Lkv)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, device=dev, dtype=torch.uint8)
    if out is not None:
        cand_idx, cand_score, cand_count = out
        assert cand_idx.is_contiguous() and cand_score.is_contiguous() and cand_count.is_contiguous()
    else:
        cand_idx = torch.zeros(R, k_eff, device=dev, dtype=torch.int32)
        cand_score = torch.empty(R, k_eff, device=dev, dtype=torch.float32)
        cand_count = torch.empty(R, device=dev, dtype=torch.int32)
    if row_stats is None:
        row_stats = torch.zeros(R, 3, device=dev, dtype=torch.float64)
    w = w.reshape(R, -1).float().contiguous()
    bias = bias.float().contiguous()
    _lib.call("gsa_indexer_select", C.byref(dims), dtype_code(qI.dtype), B, Lq, Lkv, q_pos0,
              int(causal), _p(qI), qI.stride(1), qI.stride(0), _p(kI), kI.stride(1), kI.stride(0),
              _p(w), _p(bias), float(scale), _p(shift), int(k_eff),
              _p(cand_idx), _p(cand_score), _p(cand_count), _p(row_stats), chunk_rows,
              _p(workspace), workspace.numel(), _stream())
    _after("indexer_select")
    return cand_idx, cand_score, cand_count, row_stats


SURVIVOR_CAP = 8192


def survivors_eligible(dims: Dims, k_eff: int, has_shift: bool) -> bool:
    """Whether gsa_indexer_survivors applies: sigmoid indexer with its row centre, and
    2 cap >= 3 k_eff + 2048."""
    return has_shift and dims.idx_act == ACT["sigmoid"] and 2 * SURVIVOR_CAP >= 3 * k_eff + 2048


# True (or GSA_SURVIVOR_PASS=fused in the environment): the survivor pass without the score
# matrix (gsa_indexer_survivors_fused) where it applies.  Same results, bit for bit; it moves
# 68 GB less through HBM per 128K-token forward but is slower on B200 (the survivor emission
# lengthens the indexer's issue-bound epilogue: 42.0 vs 22.3 ms, more than the streaming
# compaction it replaces), so the materialised pass is the default.
FUSED_SURVIVORS = os.environ.get("GSA_SURVIVOR_PASS", "materialised") == "fused"


def fused_survivors_eligible(dims: Dims, qI, kI) -> bool:
    """Whether gsa_indexer_survivors_fused applies: the bf16 tensor-core indexer at H_I = 8,
    d_I = 64 with 16-byte aligned qI / kI rows."""
    return (qI.dtype == torch.bfloat16 and kI.dtype == torch.bfloat16 and dims.n_idx_heads == 8
            and dims.d_idx == 64 and dims.idx_act == ACT["sigmoid"]
            and qI.data_ptr() % 16 == 0 and kI.data_ptr() % 16 == 0
            and (qI.stride(1) * 2) % 16 == 0 and (kI.stride(1) * 2) % 16 == 0
            and qI.stride(2) == 1 and kI.stride(2) == 1)


def indexer_survivors(dims: Dims, qI, kI, w, bias, scale: float, shift, k_eff: int, q_pos0: int = 0,
                      causal: bool = True, chunk_rows: int | None = None, row_stats=None, out=None,
                      fused: bool | None = None):
    """Indexer + threshold survivors for all rows, chunk by chunk.  Returns (cand_idx [R, cap],
    cand_score [R, cap], cand_count [R], row_stats): each row's candidates hold its k_eff best
    scores (and usually more), in ascending column order.  ``fused`` (default: FUSED_SURVIVORS;
    only where eligible) writes the survivors from the indexer itself instead of streaming a
    score matrix through HBM."""
    _cuda(qI, kI, w, bias, shift)
    B, Lq, _ = qI.shape
    Lkv = kI.shape[1]
    R = B * Lq
    dev = qI.device
    cap = SURVIVOR_CAP
    if fused is None:
        fused = FUSED_SURVIVORS
    fused = fused and fused_survivors_eligible(dims, qI, kI)
    global last_chunk_count, last_survivor_path
    last_survivor_path = "fused" if fused else "materialised"
    chunk_rows, last_chunk_count = _chunking(B, Lq, Lkv, chunk_rows)
    if fused:
        ws_bytes = _lib.lib().gsa_survivors_fused_workspace_size(chunk_rows, Lkv, int(k_eff), cap)
    else:
        ws_bytes = _lib.lib().gsa_survivors_workspace_size(chunk_rows, Lkv)
    workspace = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    if out is not None:
        cand_idx, cand_score, cand_count = out
        assert cand_idx.is_contiguous() and cand_score.is_contiguous() and cand_count.is_contiguous()
    else:
        cand_idx = torch.empty(R, cap, device=dev, dtype=torch.int32)
        cand_score = torch.empty(R, cap, device=dev, dtype=torch.float32)
        cand_count = torch.empty(R, device=dev, dtype=torch.int32)
    if row_stats is None:
        row_stats = torch.zeros(R, 3, device=dev, dtype=torch.float64)
    w = w.reshape(R, -1).float().contiguous()
    bias = bias.float().contiguous()
    _lib.call("gsa_indexer_survivors_fused" if fused else "gsa_indexer_survivors", C.byref(dims),
              dtype_code(qI.dtype), B, Lq, Lkv, q_pos0, int(causal),
              _p(qI), qI.stride(1), qI.stride(0), _p(kI), kI.stride(1), kI.stride(0), _p(w), _p(bias),
              float(scale), _p(shift), int(k_eff), cap, _p(cand_idx), _p(cand_score), _p(cand_count),
              _p(row_stats), chunk_rows, _p(workspace), ws_bytes, _stream())
    _after("indexer_survivors")
    return cand_idx, cand_score, cand_count, row_stats
