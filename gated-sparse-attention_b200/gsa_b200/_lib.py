"""ctypes binding of libgsa_b200.so (the C ABI declared in include/gsa_b200.h).

The library is loaded lazily on first use.  There is no fallback: if the shared library is
missing or fails to load, every GSA op raises.
"""

from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("GSA_B200_LIB", _HERE / "libgsa_b200.so"))

GSA_OK = 0
STATUS_NAMES = {
    1: "GSA_ERR_BAD_ARG",
    2: "GSA_ERR_UNSUPPORTED",
    3: "GSA_ERR_WORKSPACE",
    4: "GSA_ERR_TIMEOUT",
    5: "GSA_ERR_LAUNCH",
    6: "GSA_ERR_INDEX",
    7: "GSA_ERR_CUDA",
}
DTYPE_F32, DTYPE_BF16 = 0, 1
ACT = {"sigmoid": 0, "tanh": 1, "silu": 2, "relu": 3}


class GSAError(RuntimeError):
    """A nonzero status returned by the GSA C ABI."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed with {STATUS_NAMES.get(status, status)}")


class Dims(C.Structure):
    _fields_ = [("d_model", C.c_int32), ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32),
                ("d_head", C.c_int32), ("n_idx_heads", C.c_int32), ("d_idx", C.c_int32),
                ("gate_act", C.c_int32), ("idx_act", C.c_int32)]


class ProjLayout(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("q", "k", "v", "g2", "g1", "qi", "ki", "wi")]


class TopkParams(C.Structure):
    _fields_ = [("k_base", C.c_int32), ("k_min", C.c_int32), ("k_max", C.c_int32),
                ("use_adaptive", C.c_int32), ("temperature", C.c_float)]


P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int32
F32 = C.c_float
INT = C.c_int

# name -> argtypes (restype int unless listed in _RESTYPES)
SIGNATURES = {
    "gsa_get_device_error": [P, P],
    "gsa_version": [],
    "gsa_proj_epilogue": [P, P, INT, I64, P, I64, P, P, P, INT, I64, P, P, P, I64, P, P, P, P],
    "gsa_proj_epilogue_cache": [P, P, INT, I64, I64, P, I64, P, P, P, INT, I64, P, P, P, I64, I64, P, I64, I64,
                                P, P, P, P],
    "gsa_indexer_scores": [P, INT, I64, I64, I64, I64, INT, INT, P, I64, I64, P, I64, I64, P, P, F32,
                           P, P, I64, P, P],
    "gsa_row_stats": [I64, I64, P, I64, P, P],
    "gsa_row_summary": [I64, I64, P, I64, INT, P, P],
    "gsa_topk_candidates": [I64, I64, I64, I64, INT, P, I64, P, P, I32, P, P, P, P],
    "gsa_row_variance": [I64, I64, INT, P, P, P, P, P],
    "gsa_adaptive_k": [I64, I64, INT, P, P, P, P, P, P],
    "gsa_select_finalize": [I64, I32, P, P, P, P, P, I64, P, P, P],
    "gsa_sparse_sdpa": [P, INT, I64, I64, I64, P, P, P, I64, P, I64, P, P, P, F32, P],
    "gsa_sparse_sdpa_strided": [P, INT, I64, I64, I64, P, P, P, I64, I64, P, I64, P, P, P, F32, P, I64, P],
    "gsa_sdpa_workspace_size": [P, I64, I64],
    "gsa_add_rmsnorm": [INT, I64, I64, P, I64, P, I64, P, F32, P, I64, P, I64, P],
    "gsa_silu_mul": [INT, I64, I64, P, I64, P, I64, P],
    "gsa_sparse_sdpa_lse": [P, INT, I64, I64, I64, P, P, P, I64, I64, P, I64, P, P, P, P, F32, P],
    "gsa_sparse_sdpa_backward": [P, INT, I64, I64, I64, P, P, P, I64, I64, P, I64, P, P, P, P, P, P, P, I64, I64,
                                 F32, P],
    "gsa_decode_workspace_size": [P, P, INT, I64, I64, I64],
    "gsa_decode_attend": [P, P, P, INT, I64, I64, I64, P, I64, P, P, P, INT, I64, P, I64, P, I64, P, F32, F32, P, P,
                          P, INT, P, I64, P],
    "gsa_workspace_size": [I64, I64],
    "gsa_indexer_select": [P, INT, I64, I64, I64, I64, INT, P, I64, I64, P, I64, I64, P, P, F32, P,
                           I32, P, P, P, P, I64, P, I64, P],
    "gsa_apply_gate": [INT, INT, I64, P, P, P, P, P],
    "gsa_survivors_workspace_size": [I64, I64],
    "gsa_indexer_survivors": [P, INT, I64, I64, I64, I64, INT, P, I64, I64, P, I64, I64, P, P, F32, P,
                              I32, I32, P, P, P, P, I64, P, I64, P],
    "gsa_survivors_fused_workspace_size": [I64, I64, I32, I32],
    "gsa_indexer_survivors_fused": [P, INT, I64, I64, I64, I64, INT, P, I64, I64, P, I64, I64, P, P, F32, P,
                                    I32, I32, P, P, P, P, I64, P, I64, P],
    "gsa_indexer_select_static": [P, INT, I64, I64, I64, I64, INT, P, I64, I64, P, I64, I64, P, P, F32,
                                  P, I32, P, P, P, P, P],
    "gsa_sparse_sdpa_probs": [P, INT, I64, I64, I64, P, P, I64, I64, P, P, I64, I64, P, F32, P, P],
    "gsa_selftest_bounded_wait": [C.c_uint32, P],
    "gsa_proj_fused_rows": [P],
    "gsa_proj_fused": [P, INT, I64, I64, P, I64, P, P, P, I64, P, P, INT, I64, P, P, P, I64, I64, P, P, I64, P, I64,
                       I64, P, P, P],
}
_RESTYPES = {"gsa_version": C.c_char_p, "gsa_workspace_size": C.c_int64,
             "gsa_survivors_workspace_size": C.c_int64, "gsa_sdpa_workspace_size": C.c_int64,
             "gsa_survivors_fused_workspace_size": C.c_int64,
             "gsa_decode_workspace_size": C.c_int64, "gsa_proj_fused_rows": C.c_int64}

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (raises if it cannot be loaded)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"GSA CUDA library not found at {LIB_PATH}; build it with "
                        "`python gated-sparse-attention_b200/csrc/build.py`")
                handle = C.CDLL(str(LIB_PATH))
                for name, args in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.argtypes = args
                    fn.restype = _RESTYPES.get(name, C.c_int)
                _lib = handle
    return _lib


def call(name: str, *args) -> int:
    """Call an entry point and raise GSAError on a nonzero status."""
    st = getattr(lib(), name)(*args)
    if st != GSA_OK:
        raise GSAError(name, st)
    return st


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
