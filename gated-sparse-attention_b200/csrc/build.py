"""Build libgsa_b200.so (sm_100a) in-tree with nvcc.

Each .cu file is compiled to an object in parallel, then linked into
``gated-sparse-attention_b200/gsa_b200/libgsa_b200.so`` next to the Python package that loads
it.  Run directly (``python gated-sparse-attention_b200/csrc/build.py``) or through
``__graft_entry__.build()``.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG_ROOT = CSRC.parent
REPO = PKG_ROOT.parent
OUT_DIR = PKG_ROOT / "gsa_b200"
LIB = OUT_DIR / "libgsa_b200.so"
OBJ_DIR = PKG_ROOT / "_build"

SOURCES = ["abi.cu", "proj_epilogue.cu", "indexer_simt.cu", "indexer_tc.cu", "indexer_decode.cu", "topk.cu",
           "sparse_sdpa.cu", "sparse_sdpa_bwd.cu", "select_static.cu", "decoder.cu", "sdpa_probs.cu", "selftest.cu",
           "proj_gemm.cu"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _flags() -> list[str]:
    return ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                   f"-I{CSRC}", f"-I{REPO / 'include'}"]


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool, ptxas_v: bool) -> str:
    cmd = [nvcc, *_flags(), "-c", str(src), "-o", str(obj)]
    if ptxas_v:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return res.stderr if (verbose or ptxas_v) else ""


def build(verbose: bool = False, ptxas_v: bool = False, force: bool = False) -> Path:
    nvcc = _nvcc()
    OBJ_DIR.mkdir(exist_ok=True)
    srcs = [CSRC / s for s in SOURCES if (CSRC / s).exists()]
    headers = list(CSRC.glob("*.cuh")) + [REPO / "include" / "gsa_b200.h"]
    newest_header = max(h.stat().st_mtime for h in headers)
    jobs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for src in srcs:
            obj = OBJ_DIR / (src.stem + ".o")
            stale = (force or not obj.exists() or obj.stat().st_mtime < src.stat().st_mtime
                     or obj.stat().st_mtime < newest_header)
            if stale or ptxas_v:
                jobs.append((src, ex.submit(_compile, nvcc, src, obj, verbose, ptxas_v)))
        for src, fut in jobs:
            log = fut.result()
            if log:
                print(f"--- {src.name}\n{log}", file=sys.stderr)
    objs = [str(OBJ_DIR / (s.stem + ".o")) for s in srcs]
    if jobs or not LIB.exists():
        cmd = [nvcc, *ARCH, "-shared", "-o", str(LIB), *objs, "-lcudart", "-lcuda"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_v="--ptxas" in sys.argv, force="--force" in sys.argv))
