"""The C ABI library loads and exports every entry point include/gsa_b200.h declares (CPU only:
no entry point that touches the GPU is called)."""

import ctypes
import re

from conftest import ROOT

HEADER = ROOT / "include" / "gsa_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char\s*\*)\s+(gsa_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "gsa_sparse_sdpa" in names and "gsa_indexer_select" in names
    assert len(names) >= 12


def test_library_exports_every_declared_symbol():
    from gsa_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in gsa_b200.h but not exported"


def test_binding_covers_header():
    from gsa_b200 import _lib

    assert sorted(_lib.exported_symbols()) == declared_functions()


def test_version_and_workspace_without_gpu():
    from gsa_b200 import _lib

    lib = _lib.lib()
    assert b"sm_100a" in lib.gsa_version()
    assert lib.gsa_workspace_size(128, 1000) == 128 * 1000 * 4
    assert lib.gsa_workspace_size(3, 5) == 3 * 8 * 4
    assert lib.gsa_workspace_size(0, 5) == 0


def test_bad_arguments_are_rejected_before_any_launch():
    """Argument validation returns GSA_ERR_BAD_ARG without touching the device."""
    from gsa_b200 import _lib

    lib = _lib.lib()
    # negative sizes / null pointers
    assert lib.gsa_topk_candidates(-1, 1, 10, 0, 0, None, 10, None, None, 4, None, None, None, None) == 1
    assert lib.gsa_topk_candidates(4, 4, 10, 0, 0, None, 10, None, None, 0, None, None, None, None) == 1
    assert lib.gsa_select_finalize(4, 8, None, None, None, None, None, 4, None, None, None) == 1
    assert lib.gsa_row_stats(4, 10, None, 5, None, None) == 1
    assert lib.gsa_apply_gate(7, 0, 10, None, None, None, None, None) == 1
    # empty work is a no-op success
    assert lib.gsa_topk_candidates(0, 1, 10, 0, 0, None, 10, None, None, 4, None, None, None, None) == 0


def test_survivor_entry_points_validate_before_any_launch():
    """gsa_indexer_survivors / gsa_survivors_workspace_size / gsa_select_finalize reject bad
    arguments without touching the device (CPU only)."""
    import ctypes as C

    from gsa_b200 import _lib, ops

    lib = _lib.lib()
    ld = (1000 + 3) // 4 * 4
    # score scratch, failed rows, their count, segment counts, the indexer's per-key-range
    # statistic partials (16 rows x 1 range of 32 key tiles x 3 doubles)
    assert lib.gsa_survivors_workspace_size(16, 1000) == ((16 * ld * 4 + 255) // 256) * 256 + 256 + 256 + 1024 + 512
    assert lib.gsa_survivors_workspace_size(0, 1000) == 0
    dims = ops.make_dims(4096, 32, 8, 128, 8, 64)
    relu = ops.make_dims(4096, 32, 8, 128, 8, 64, idx_act="relu")
    p = C.c_void_p(16)  # a stand-in pointer: every case below returns before using it

    def call(d, k_eff, cap, shift=p, ws_bytes=1 << 40, chunk=16):
        return lib.gsa_indexer_survivors(C.byref(d), 1, 1, 100, 1000, 0, 1, p, 512, 0, p, 64, 0, p, p, 0.125,
                                         shift, k_eff, cap, p, p, p, p, chunk, p, ws_bytes, None)

    assert call(dims, 0, 8192) == 1                 # k_eff < 1
    assert call(dims, 4096, 1024) == 1              # cap < k_eff
    assert call(dims, 64, 8192, shift=None) == 1    # the row centre is required
    assert call(dims, 64, 8192, chunk=0) == 1       # no chunk rows
    assert call(relu, 64, 8192) == 2                # thresholds need the sigmoid indexer
    assert call(dims, 6000, 8192) == 2              # no room above 1.5 k_eff in the cap
    assert call(dims, 64, 8192, ws_bytes=100) == 3  # workspace too small
    # empty work is a no-op success
    assert lib.gsa_indexer_survivors(C.byref(dims), 1, 1, 0, 1000, 0, 1, p, 512, 0, p, 64, 0, p, p, 0.125, p,
                                     64, 8192, p, p, p, p, 16, p, 1 << 40, None) == 0
    assert lib.gsa_select_finalize(4, 0, p, p, p, p, p, 4, p, None, None) == 1   # k_eff < 1
    assert lib.gsa_select_finalize(4, 8, p, p, p, p, p, 0, p, None, None) == 1   # sel_ld < 1


def test_fused_survivor_entry_points_validate_before_any_launch():
    """gsa_survivors_fused_workspace_size against its layout restated here (the segment area
    brute-forced over every row length), and gsa_indexer_survivors_fused rejecting bad arguments
    without touching the device (CPU only)."""
    import ctypes as C

    from gsa_b200 import _lib, ops

    lib = _lib.lib()
    a256 = lambda x: (x + 255) // 256 * 256

    def seg_cap(n, K, cap):
        if n <= cap:
            return 4096
        c = (4 * 4096 * ((14 * K + 9) // 10) + n - 1) // n
        return min(4096, (c + 31) // 32 * 32 + 128)

    for chunk, n_cols, K, cap in [(16, 1000, 64, 8192), (8192, 131072, 4096, 8192), (300, 50000, 1024, 4096)]:
        stride = max((n + 4095) // 4096 * seg_cap(n, K, cap) for n in range(1, n_cols + 1))
        ranges = (n_cols + 4095) // 4096
        want = (lib.gsa_survivors_workspace_size(chunk, n_cols) + a256(chunk * 24) + a256(chunk * ranges * 4)
                + 2 * a256(chunk * stride * 4) + a256(chunk * 4 + 4))
        assert lib.gsa_survivors_fused_workspace_size(chunk, n_cols, K, cap) == want, (chunk, n_cols, K, cap)
    assert lib.gsa_survivors_fused_workspace_size(0, 1000, 64, 8192) == 0
    assert lib.gsa_survivors_fused_workspace_size(16, 1000, 0, 8192) == 0
    assert lib.gsa_survivors_fused_workspace_size(16, 1000, 64, 32) == 0

    dims = ops.make_dims(4096, 32, 8, 128, 8, 64)
    relu = ops.make_dims(4096, 32, 8, 128, 8, 64, idx_act="relu")
    hi4 = ops.make_dims(4096, 32, 8, 128, 4, 64)
    p = C.c_void_p(16)  # a stand-in pointer: every case below returns before using it

    def call(d, k_eff, cap, shift=p, ws_bytes=1 << 40, chunk=16, B=1, Lq=100):
        return lib.gsa_indexer_survivors_fused(C.byref(d), 1, B, Lq, 1000, 0, 1, p, 512, 0, p, 64, 0, p, p, 0.125,
                                               shift, k_eff, cap, p, p, p, p, chunk, p, ws_bytes, None)

    assert call(dims, 0, 8192) == 1                 # k_eff < 1
    assert call(dims, 4096, 1024) == 1              # cap < k_eff
    assert call(dims, 64, 8192, shift=None) == 1    # the row centre is required
    assert call(dims, 64, 8192, chunk=0) == 1       # no chunk rows
    assert call(dims, 64, 8192, B=-1) == 1
    assert call(relu, 64, 8192) == 2                # thresholds need the sigmoid indexer
    assert call(hi4, 64, 8192) == 2                 # the emitting indexer takes 8 heads
    assert call(dims, 6000, 8192) == 2              # no room above 1.5 k_eff in the cap
    assert call(dims, 64, 8192, ws_bytes=100) == 3  # workspace too small
    assert call(dims, 64, 8192, Lq=0) == 0          # empty work is a no-op success


def test_fused_survivor_eligibility():
    """ops.fused_survivors_eligible mirrors the C side's checks: bf16 q^I / k^I, 8 indexer heads
    of 64, the sigmoid indexer, 16-byte aligned rows with a contiguous last dimension (CPU only)."""
    import torch

    from gsa_b200 import ops

    dims = ops.make_dims(4096, 32, 8, 128, 8, 64)
    qI = torch.zeros(1, 64, 512, dtype=torch.bfloat16)
    kI = torch.zeros(1, 64, 64, dtype=torch.bfloat16)
    assert ops.fused_survivors_eligible(dims, qI, kI)
    assert not ops.fused_survivors_eligible(dims, qI.float(), kI.float())
    assert not ops.fused_survivors_eligible(ops.make_dims(4096, 32, 8, 128, 4, 64), qI[..., :256], kI)
    assert not ops.fused_survivors_eligible(ops.make_dims(4096, 32, 8, 128, 8, 64, idx_act="relu"), qI, kI)
    assert not ops.fused_survivors_eligible(dims, qI, torch.zeros(1, 64, 65, dtype=torch.bfloat16)[..., 1:])
    # a switch the caller can flip: the materialised pass unless asked otherwise
    assert isinstance(ops.FUSED_SURVIVORS, bool)


def test_cache_entry_points_validate_before_any_launch():
    """gsa_proj_epilogue_cache and gsa_sparse_sdpa_strided reject a batch stride that cannot
    hold the sequence, without touching the device (CPU only)."""
    import ctypes as C

    from gsa_b200 import _lib, ops

    lib = _lib.lib()
    dims = ops.make_dims(4096, 32, 8, 128, 8, 64)
    lay = _lib.ProjLayout(0, 4096, 5120, 6144, 7168, 11264, 11776, 11840)
    p = C.c_void_p(16)  # a stand-in pointer: every case below returns before using it
    kv_ld = 2 * 8 * 128

    def epi(B, L, kv_bstride, ki=None, ki_ld=64, ki_bstride=1 << 30):
        return lib.gsa_proj_epilogue_cache(C.byref(dims), C.byref(lay), 1, B, L, p, 15936, p, p, p, 1, 4096, p, p,
                                           p, kv_ld, kv_bstride, ki, ki_ld, ki_bstride, p, p, p, None)

    assert epi(2, 10, 9 * kv_ld) == 1                            # batch stride below L rows
    assert epi(2, 10, 10 * kv_ld, ki=p, ki_ld=32) == 1           # k^I rows narrower than d_I
    assert epi(2, 10, 10 * kv_ld, ki=p, ki_bstride=9 * 64) == 1  # k^I batch stride below L rows
    assert epi(2, 0, 0) == 0 and epi(0, 10, 0) == 0              # empty work is a no-op success

    def sdpa(Lkv, kv_bstride):
        return lib.gsa_sparse_sdpa_strided(C.byref(dims), 1, 2, 1, Lkv, p, p, p, kv_ld, kv_bstride, p, 16, p, None,
                                           p, 0.1, None, 0, None)

    assert sdpa(100, 99 * kv_ld) == 1
    assert lib.gsa_sparse_sdpa_strided(C.byref(dims), 1, 0, 1, 100, p, p, p, kv_ld, 100 * kv_ld, p, 16, p, None, p,
                                       0.1, None, 0, None) == 0


def test_training_and_decoder_entry_points_validate_before_any_launch():
    """gsa_sparse_sdpa_lse, gsa_sparse_sdpa_backward, gsa_add_rmsnorm and gsa_silu_mul reject bad
    arguments without touching the device (CPU only)."""
    import ctypes as C

    from gsa_b200 import _lib, ops

    lib = _lib.lib()
    dims = ops.make_dims(4096, 32, 8, 128, 8, 64)
    p = C.c_void_p(256)  # a stand-in pointer: every case below returns before using it
    kv_ld = 2 * 8 * 128
    # lse output is required
    assert lib.gsa_sparse_sdpa_lse(C.byref(dims), 1, 1, 4, 100, p, p, p, kv_ld, 100 * kv_ld, p, 16, p, None, p, None,
                                   0.1, None) == 1

    def bwd(dtype=1, kv_bstride=100 * kv_ld, dkv_ld=1024, dkv_bstride=100 * 1024, dq=p):
        return lib.gsa_sparse_sdpa_backward(C.byref(dims), dtype, 1, 4, 100, p, p, p, kv_ld, kv_bstride, p, 16, p, p,
                                            p, p, dq, p, p, dkv_ld, dkv_bstride, 0.1, None)

    assert bwd(dtype=7) == 1                   # unknown dtype
    assert bwd(kv_bstride=99 * kv_ld) == 1     # batch stride below the keys
    assert bwd(dkv_ld=512) == 1                # gradient rows narrower than Hk * D
    assert bwd(dq=None) == 1                   # dq required
    # decoder-layer elementwise ops
    assert lib.gsa_add_rmsnorm(1, 4, 0, p, 8, None, 0, p, 1e-5, None, 0, p, 8, None) == 1       # d < 1
    assert lib.gsa_add_rmsnorm(1, 4, 8, p, 8, None, 0, p, 1e-5, p, 8, p, 8, None) == 1          # h_out without a
    assert lib.gsa_add_rmsnorm(1, 4, 8, p, 8, None, 0, None, 1e-5, None, 0, p, 8, None) == 1    # y_out without w
    assert lib.gsa_add_rmsnorm(1, 0, 8, None, 8, None, 0, None, 1e-5, None, 0, None, 8, None) == 0  # empty
    assert lib.gsa_silu_mul(1, 4, 8, p, 15, p, 8, None) == 1    # gu row shorter than 2n
    assert lib.gsa_silu_mul(1, 0, 8, None, 16, None, 8, None) == 0


def test_static_select_checks_arguments_before_writing_row_stats():
    """gsa_indexer_select_static zeroes row_stats itself, but only after every argument check:
    a call that returns an error leaves the caller's buffer as it was (CPU only: the buffer is
    host memory and nothing reaches the device)."""
    import ctypes as C

    from gsa_b200 import _lib, ops

    lib = _lib.lib()
    good = ops.make_dims(4096, 32, 8, 128, 8, 64)
    bad = ops.make_dims(4096, 32, 8, 128, 8, 64)
    bad.n_kv_heads = 5  # 32 heads do not group over 5 KV heads
    p = C.c_void_p(256)  # a stand-in device pointer: every case below returns before using it
    stats = (C.c_double * 12)(*([7.5] * 12))

    def call(d, dtype=1, qI=p, k_eff=16, cand=p):
        return lib.gsa_indexer_select_static(C.byref(d), dtype, 1, 4, 100, 0, 1, qI, 512, 0, p, 64, 0, p, p,
                                             0.125, p, k_eff, cand, p, p, stats, None)

    assert call(bad) == 1            # dims that no kernel takes
    assert call(good, dtype=9) == 1  # unknown dtype
    assert call(good, qI=None) == 1  # missing indexer queries
    assert call(good, k_eff=0) == 1  # k_eff < 1
    assert call(good, cand=None) == 1
    assert list(stats) == [7.5] * 12, "row_stats was written by a call that failed its checks"


def test_probability_and_diagnostic_entry_points_validate_before_any_launch():
    """gsa_sparse_sdpa_probs and gsa_selftest_bounded_wait reject bad arguments on the host (CPU only)."""
    import ctypes as C

    from gsa_b200 import _lib, ops

    lib = _lib.lib()
    dims = ops.make_dims(512, 8, 2, 64, 4, 32)
    p = C.c_void_p(256)  # a stand-in pointer: every case below returns before using it

    def probs(B=1, Lq=4, k_eff=16, idx_ld=16, kv_ld=256, kv_bstride=100 * 256, q=p):
        return lib.gsa_sparse_sdpa_probs(C.byref(dims), 1, B, Lq, 100, q, p, kv_ld, kv_bstride, p, None, idx_ld,
                                         k_eff, p, 0.125, p, None)

    assert probs(idx_ld=8) == 1               # candidate rows shorter than k_eff
    assert probs(kv_ld=64) == 1               # key rows narrower than Hk * D
    assert probs(kv_bstride=99 * 256) == 1    # batch stride below the keys
    assert probs(q=None) == 1
    assert probs(B=2, Lq=40000) == 1          # more rows than an analysis output takes
    assert probs(Lq=0) == 0 and probs(k_eff=0) == 0
    assert lib.gsa_selftest_bounded_wait(0, None) == 1   # a zero poll limit is refused, nothing launched


def test_header_is_plain_c_and_a_c_program_links():
    """A C99 program includes gsa_b200.h (no CUDA or torch headers needed), links the library and
    calls the entry points that touch no GPU; the header also compiles as C++."""
    import shutil
    import subprocess

    import pytest

    from gsa_b200 import _lib

    if shutil.which("gcc") is None or shutil.which("g++") is None:
        pytest.skip("no host C compiler")
    out = ROOT / "tests" / "_build" / "c_abi"
    out.mkdir(parents=True, exist_ok=True)
    src = out / "use.c"
    src.write_text('#include "gsa_b200.h"\n#include <stdio.h>\n'
                   "int main(void) {\n  puts(gsa_version());\n"
                   "  return gsa_workspace_size(2, 8) == 64 ? 0 : 1;\n}\n")
    lib = _lib.LIB_PATH
    exe = out / "use"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"), str(src),
                    str(lib), f"-Wl,-rpath,{lib.parent}", "-o", str(exe)], check=True)
    p = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert p.returncode == 0 and "sm_100a" in p.stdout
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-fsyntax-only", "-x", "c++", "-I",
                    str(ROOT / "include"), str(src)], check=True)
