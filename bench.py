"""GSA layer forward throughput on B200 (tokens/s), 128K-context workload.

Workload (one "step"): one GatedSparseAttention forward, d_model 4096, 32 query / 8 KV heads of
128, 8 indexer heads of 64, k_base 2048 (k_min 256, k_max 4096, adaptive), value and output gates
on, bf16, batch 1 x 131072 tokens, x ~ N(0,1), weights from the default init with seed 0.
With N > 1 GPUs (torchrun) the query sequence is sharded: it is cut into 2N segments and rank r
owns segments r and 2N-1-r (equal causal work per rank); K / V / indexer keys are all-gathered
over NCCL and the adaptive-k variance sum is all-reduced; ``value`` is 131072 / (max over ranks
of the step time).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--seq-len L]

``--impl reference`` times the reference algorithm's CPU path (the oracle restatement of the
reference's PyTorch ops, oracle/gsa_oracle.py) on the host cores, sampled and extrapolated.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "gated-sparse-attention_b200"))

import torch  # noqa: E402

ZIGZAG_FOLDS = 4  # query layout across ranks (gsa_b200.sharded): 2 x folds segments per rank
WORKLOAD = dict(d_model=4096, n_heads=32, n_kv_heads=8, d_indexer=64, n_indexer_heads=8,
                k_base=2048, k_min=256, k_max=4096)
# prefill shapes of the 4096-wide layer (batch, tokens per sequence, k clamps): the 128K headline
# sequence, the README quickstart batch (two 8192-token sequences whose adaptive-k variance mean
# spans both) and one 32768-token sequence with k clipped to [512, 4096]
PREFILL_SHAPES = {"prefill": (1, 131072, 256, 4096), "c2": (2, 8192, 256, 4096), "c3": (1, 32768, 512, 4096)}
METRIC = "GSA layer fwd tokens/sec at 128K ctx (1/2/4/8 B200); % HBM / tensor roofline"
PREFILL_METRIC = "GSA layer fwd tokens/sec (B200)"


def prefill_workload_name(B, L, k_min, k_max):
    return f"GSA layer fwd B={B} L={L} d4096 h32/8x128 idx8x64 k2048[{k_min},{k_max}] bf16"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


_RESULT_FD = None


def quiet_stdout():
    """Send everything written to stdout (NCCL's version banner, library prints) to stderr at
    the file-descriptor level, keeping a handle on the real stdout for the one result line."""
    global _RESULT_FD
    if _RESULT_FD is None:
        sys.stdout.flush()
        _RESULT_FD = os.dup(1)
        os.dup2(2, 1)


def emit(res: dict):
    line = (json.dumps(res) + "\n").encode()
    if _RESULT_FD is None:
        sys.stdout.write(line.decode())
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, line)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# ---------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_ms: int = 50):
        self.gpu = gpu_index
        self.period_ms = period_ms
        self.proc = None
        self.lines = []
        self.skip = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.period_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi takes a while to start: wait for its first sample, so that the sampling
            # loop is running when the timed region begins, and count only the samples after it
            t0 = time.time()
            while not self.lines and self.proc.poll() is None and time.time() - t0 < 5.0:
                time.sleep(0.01)
            self.skip = len(self.lines)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[self.skip:]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
# distributed helpers
# ---------------------------------------------------------------------------------------------
def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------
def sdpa_algorithmic_bytes(cfg, cnt: torch.Tensor) -> float:
    """Bytes the sparse SDPA must move: the gathered K and V rows (Hk*D bf16 each per selected
    key), q / gate read and out write (H*D bf16 each per row), and the int32 indices."""
    Hk, H, D = cfg.n_kv_heads, cfg.n_heads, cfg.d_head
    sum_k = float(cnt.double().sum().item())
    rows = cnt.numel()
    return sum_k * (2 * Hk * D * 2 + 4) + rows * 3 * H * D * 2


def causal_pairs(first: int, m: int, n_keys: int) -> int:
    """Sum over query positions first .. first + m - 1 of the keys each sees, min(n_keys, pos + 1)."""
    m1 = min(m, max(0, n_keys - first))          # rows not yet clipped by n_keys
    return m1 * (first + 1) + m1 * (m1 - 1) // 2 + (m - m1) * n_keys


def indexer_roofline(cap, cfg, pk, chunk_bytes=4 << 30, reps=2):
    """The tensor-core indexer timed alone over this rank's query segments (the forward's own
    q^I, k^I, w), chunked like the layer, scores into one reused scratch: algorithmic flops
    2*H_I*d_I per causal (query, key) pair against the measured bf16 GEMM peak, and its sigmoid
    (tanh) rate against the MUFU pipe's 16 results / clock / SM at the maximum SM clock."""
    import ctypes as C
    from gsa_b200 import _lib, ops

    qI, kI, w, shift = cap["qI"], cap["kI"], cap["w"], cap["shift"]
    dims, HI, dI = cap["dims"], cfg.n_indexer_heads, cfg.d_indexer
    B, Lkv = qI.shape[0], kI.shape[1]
    ld = (Lkv + 3) // 4 * 4
    rows_max = max(1, chunk_bytes // (4 * ld))
    scratch = torch.empty(min(rows_max, max(n for _, n, _ in cap["idx_segments"])) * ld, device=qI.device,
                          dtype=torch.float32)
    wv = w.reshape(-1, HI).float().contiguous()
    bias = cap["bias"].float().contiguous()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    pairs = 0
    launches = []
    for l0, n, p0 in cap["idx_segments"]:
        for t0 in range(0, n, rows_max):
            m = min(rows_max, n - t0)
            q = qI[:, l0 + t0:l0 + t0 + m]
            launches.append((q, m, p0 + t0, l0 + t0))
            pairs += causal_pairs(p0 + t0, m, Lkv)
    pairs = pairs * B

    def run():
        for q, m, qpos, r0 in launches:
            _lib.call("gsa_indexer_scores", C.byref(dims), ops.dtype_code(q.dtype), 1, m, Lkv, qpos, 1, 0,
                      C.c_void_p(q.data_ptr()), q.stride(1), 0, C.c_void_p(kI.data_ptr()), kI.stride(1), 0,
                      C.c_void_p(wv[r0:].data_ptr()), C.c_void_p(bias.data_ptr()), float(cap["idx_scale"]),
                      C.c_void_p(shift[r0:].data_ptr()), C.c_void_p(scratch.data_ptr()), ld, None, stream)

    run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = 2.0 * HI * dI * pairs
    achieved = flops / (ms / 1e3) / 1e12
    tanh_peak = 148 * 16 * pk.get("sm_max_mhz", 1965.0) * 1e6
    tanh_rate = HI * pairs / (ms / 1e3)
    return {"kernel": "gsa::tc::indexer_tc_kernel<8, 0>", "bound": "tensor", "achieved": round(achieved, 1),
            "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": round(achieved / pk["bf16_tflops"], 4),
            "algorithmic_flops": flops, "kernel_ms": round(ms, 3), "launches": len(launches),
            "epilogue": {"bound": "mufu", "tanh_per_s": tanh_rate, "peak_tanh_per_s": tanh_peak,
                         "frac": round(tanh_rate / tanh_peak, 4),
                         "note": "H_I sigmoids per pair, one tanh.approx each; 16 per clock per SM at the "
                                 "maximum SM clock"}}


def proj_roofline(m, x, pk, reps=3):
    """The fused projection GEMM (all projections + RoPE, G2, G1 gate, q^I / k^I, w in its epilogue)
    timed alone on this rank's input: algorithmic flops 2 * T * d_model * N (N = the regrouped
    weight rows) against the measured bf16 GEMM peak, and the bytes it must move (x and the
    weights read, its outputs written) against the HBM peak.  None when the layer does not take
    the fused path (fp32, or shapes it declines)."""
    from gsa_b200 import ops

    B, L, d = x.shape
    dims = m._step_constants()[0]
    Wp, bp = m.fused_projection_tiles()
    sp = m.query_shards
    pos = (sp.positions(L, x.device) if sp is not None else torch.arange(L, device=x.device)).unsqueeze(0)
    pos = pos.expand(B, -1)
    xs = x.reshape(B * L, d)

    def run():
        return ops.proj_fused(dims, Wp, bp, xs, B, L, pos, m.rotary_emb.cos_cached, m.rotary_emb.sin_cached)

    with torch.no_grad():
        if run() is None:
            return None
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            run()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    cfg = m.config
    T, N = B * L, Wp.shape[0]
    flops = 2.0 * T * d * N
    H, Hk, D, HI, dI = cfg.n_heads, cfg.n_kv_heads, m.d_head, cfg.n_indexer_heads, cfg.d_indexer
    out_bytes = T * ((2 * H * D + 2 * Hk * D + HI * dI + dI) * 2 + 4 * (HI + 1))
    nbytes = T * d * 2 + N * d * 2 + out_bytes
    achieved = flops / (ms / 1e3) / 1e12
    return {"kernel": "pg::proj_gemm_kernel", "bound": "tensor", "achieved": round(achieved, 1),
            "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": round(achieved / pk["bf16_tflops"], 4),
            "algorithmic_flops": flops, "kernel_ms": round(ms, 3),
            "bytes": nbytes, "hbm_frac": round(nbytes / (ms / 1e3) / 1e9 / pk["hbm_gbs"], 4),
            "note": "timed alone (3 launches); the peak is the measured cuBLAS bf16 burst figure"}


SDPA_TRAFFIC = ROOT / "profiles" / "sparse_sdpa_traffic.json"
SDPA_SOURCE = ROOT / "gated-sparse-attention_b200" / "csrc" / "sparse_sdpa.cu"


def source_sha(path: Path) -> str:
    import hashlib

    return hashlib.sha256(path.read_bytes()).hexdigest()[:16]


def sdpa_dram_traffic(workload: str, B: int, L: int, world: int, sdpa_bytes: float):
    """DRAM bytes (read + write) of one SDPA launch from the committed ncu capture of this workload
    (profiles/sparse_sdpa_traffic.json: one entry per captured shape, each with the sha of the
    kernel source it was captured from).  Returns (bytes or None, note)."""
    if not SDPA_TRAFFIC.exists():
        return None, "no ncu capture committed"
    caps = json.loads(SDPA_TRAFFIC.read_text()).get("captures", [])
    sha = source_sha(SDPA_SOURCE)
    for c in caps:
        if c["workload"] == workload and c["batch"] == B and c["seq_len"] == L:
            t = c["dram_bytes_read"] + c["dram_bytes_write"]
            note = f"ncu capture of this workload ({c['launch']})"
            if world > 1:
                # a shard's launch: the capture's DRAM bytes per algorithmic byte
                t = t / c["algorithmic_bytes"] * sdpa_bytes
                note = f"one-GPU capture of this workload scaled to the shard's algorithmic bytes ({c['launch']})"
            if c.get("source_sha") != sha:
                note += f"; captured from an earlier kernel source (sha {c.get('source_sha')}, now {sha})"
            return t, note
    return None, "no ncu capture of this workload"


def sdpa_roofline(cfg, cnt, sdpa_ms, sdpa_bytes, pk, pk_kind, clocks, dev, workload, B, L, world):
    """The SDPA's roofline.  Its binding limit is shared-memory bandwidth: every selected key's K and V
    rows (2*Hk*D bf16) are written into shared memory by a bulk copy and read back once by ldmatrix,
    against 128 B / clock / SM at the median SM clock of the timed steps -- that is ``frac``.  Beside it:
    the DRAM bytes of one launch (ncu) against the measured HBM peak, and the rate of the bytes the rows
    gather (per row its k_t K and V rows, q, gate, out, indices), which nearby rows serve from L2 and
    which therefore exceeds the DRAM peak ("l2_amplified")."""
    t = sdpa_ms / 1e3
    sm_mhz = clocks.get("sm_mhz") or pk.get("sm_max_mhz", 1965.0)
    n_sms = torch.cuda.get_device_properties(dev).multi_processor_count
    sum_k = float(cnt.double().sum().item())
    smem_bytes = sum_k * 2 * (2 * cfg.n_kv_heads * cfg.d_head * 2)
    smem_peak = 128.0 * n_sms * sm_mhz * 1e6 / 1e9
    smem_rate = smem_bytes / t / 1e9
    hbm = pk["hbm_gbs"]
    traffic, note = sdpa_dram_traffic(workload, B, L, world, sdpa_bytes)
    alg_rate = sdpa_bytes / t / 1e9
    return {"kernel": "gsa::sdpa_tc_kernel<128,4,14>", "bound": "smem", "achieved": round(smem_rate, 1),
            "peak": round(smem_peak, 1), "unit": "GB/s", "frac": round(smem_rate / smem_peak, 4),
            "peak_kind": f"128 B/clk/SM x {n_sms} SMs at the {sm_mhz:.0f} MHz median SM clock of the timed steps",
            "bytes": smem_bytes, "traffic": traffic, "traffic_note": note, "kernel_ms": round(sdpa_ms, 3),
            "mean_k": sum_k / cnt.numel(),
            "dram": (None if traffic is None else
                     {"achieved": round(traffic / t / 1e9, 1), "peak": hbm, "unit": "GB/s",
                      "frac": round(traffic / t / 1e9 / hbm, 4), "peak_kind": pk_kind}),
            "l2_amplified": {"algorithmic_bytes": sdpa_bytes, "achieved": round(alg_rate, 1), "unit": "GB/s",
                             "frac_of_hbm_peak": round(alg_rate / hbm, 4),
                             "note": "bytes the rows gather, most of them L2 hits: not a DRAM rate"}}


def prefill_shape(args):
    """(batch, tokens per sequence, k_min, k_max) of the prefill workload; --seq-len overrides L."""
    B, L, k_min, k_max = PREFILL_SHAPES[args.workload]
    return B, (args.seq_len or L), k_min, k_max


def run_ours(args, world, rank):
    from gsa_b200 import GSAConfig, GatedSparseAttention, ops
    from gsa_b200.sharded import enable_query_sharding, zigzag_slice

    dev = torch.device("cuda", torch.cuda.current_device())
    B, L, k_min, k_max = prefill_shape(args)
    cfg = GSAConfig(**{**WORKLOAD, "k_min": k_min, "k_max": k_max}, max_position_embeddings=max(131072, L))
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).eval().to(torch.bfloat16).to(dev)
    zigzag = B == 1
    if world > 1:
        import torch.distributed as dist

        # zigzag with 4 folds: 8 segments per rank dealt in alternating sweeps, which balances the
        # causal indexer work exactly and the SDPA work (k_t grows with the position) to ~2%; a
        # batch of several sequences takes contiguous blocks of every sequence
        if zigzag:
            enable_query_sharding(m, dist.group.WORLD, layout="zigzag", folds=ZIGZAG_FOLDS)
        else:
            enable_query_sharding(m, dist.group.WORLD, layout="contiguous")
    assert L % (2 * ZIGZAG_FOLDS * world) == 0
    Lr = L // world
    gen = torch.Generator().manual_seed(1)
    x_full = torch.randn(B, L, cfg.d_model, generator=gen, dtype=torch.float32)
    if world == 1:
        x_host = x_full
    elif zigzag:
        x_host = zigzag_slice(x_full, world, rank, ZIGZAG_FOLDS)
    else:
        x_host = x_full[:, rank * Lr:(rank + 1) * Lr]
    x_host = x_host.to(torch.bfloat16).contiguous().pin_memory()
    del x_full
    x = x_host.to(dev)
    torch.cuda.synchronize()

    def step():
        with torch.no_grad():
            return m(x)[0]

    # warm-up
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.check_device_error()

    # timed region (device events), clocks sampled meanwhile
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if world == 1 else int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize()
        barrier(world)
    ms_local = start.elapsed_time(end) / args.steps
    ms = max_over_ranks(ms_local, world)
    value = B * L / (ms / 1e3)

    # end to end through the public API: every step copies its x from pinned host memory and reads
    # its output back.  The copies run on a copy stream, double-buffered as a serving loop does:
    # step i+1's input goes up and step i's output comes down while the layer computes, so only the
    # first upload and the last download are exposed.
    out_host = torch.empty(B, Lr, cfg.d_model, dtype=torch.bfloat16).pin_memory()
    xd = [x, torch.empty_like(x)]
    cs = torch.cuda.current_stream(dev)
    ps = torch.cuda.Stream(dev)
    up = [torch.cuda.Event(), torch.cuda.Event()]
    barrier(world)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(cs)
    ps.wait_stream(cs)
    with torch.cuda.stream(ps):
        xd[0].copy_(x_host, non_blocking=True)
        up[0].record(ps)
    for i in range(args.steps):
        cs.wait_event(up[i % 2])
        with torch.no_grad():
            out = m(xd[i % 2])[0]
        done = torch.cuda.Event()
        done.record(cs)
        with torch.cuda.stream(ps):
            if i + 1 < args.steps:
                # xd[(i+1) % 2] was read by step i-1, which ended before step i's download below
                xd[(i + 1) % 2].copy_(x_host, non_blocking=True)
                up[(i + 1) % 2].record(ps)
            ps.wait_event(done)
            out_host.copy_(out, non_blocking=True)
            out.record_stream(ps)
        del out
    cs.wait_stream(ps)
    e1.record(cs)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    e2e = {"value": B * L / (e2e_ms / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": x_host.numel() * x_host.element_size() * world,
           "d2h_bytes_per_step": out_host.numel() * out_host.element_size() * world,
           "ms_per_step": e2e_ms,
           "copies": "pinned host <-> device every step on a copy stream, double-buffered against the "
                     "neighbouring steps' compute"}

    # stage breakdown and the SDPA kernel alone (roofline)
    cap = {}
    marks = []

    def mark(name):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        marks.append((name, ev))

    with torch.no_grad():
        e_start = torch.cuda.Event(enable_timing=True)
        e_start.record()
        m._forward_impl(x, None, None, False, False, mark=mark, capture=cap)
    torch.cuda.synchronize()
    stages, prev = {}, e_start
    for name, ev in marks:
        stages[name] = round(prev.elapsed_time(ev), 3)
        prev = ev
    shard_balance = None
    if world > 1:
        # every rank's stage times (the step waits for the slowest) and the SDPA work per rank
        import torch.distributed as dist

        names = sorted(stages)
        t = torch.tensor([stages[n] for n in names], device=dev, dtype=torch.float64)
        t_max = t.clone()
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
        stages = {n: round(float(v), 3) for n, v in zip(names, t.tolist())}
        stages_max = {n: round(float(v), 3) for n, v in zip(names, t_max.tolist())}
        keys = torch.tensor([float(cap["cnt"].double().sum())], device=dev, dtype=torch.float64)
        allk = [torch.zeros_like(keys) for _ in range(world)]
        dist.all_gather(allk, keys)
        allk = [float(v) for v in torch.cat(allk).tolist()]
        shard_balance = {"stages_ms_max_over_ranks": stages_max,
                         "sdpa_keys_busiest_over_mean": round(max(allk) / (sum(allk) / world), 4),
                         "note": "stages_ms is rank 0's; kv = the blocking k^I all-gather and the start of the "
                                 "asynchronous K/V all-gather; kv_gather_wait = the wait for K/V before the SDPA"}
    # our kernels per forward: the fused projection GEMM; per query chunk the indexer and the
    # candidate pass -- fused survivors: the sampled-statistics pass, the survivor-emitting pass, its
    # ordered statistics sum, the segment join, the failed blocks' recomputation and the exact
    # fallback; materialised survivors: the scores, the ordered statistics sum, the compaction and
    # the fallback; exact: the scores and the top-k -- row variance (2) and adaptive k; the final
    # selection; the SDPA
    n_chunks = cap["n_chunks"]
    if cap.get("candidate_path") != "survivors":
        per_chunk = 2
    else:
        per_chunk = 6 if cap.get("survivor_pass") == "fused" else 4
    launches_per_step = 1 + per_chunk * n_chunks + (3 if cfg.use_adaptive_k else 1) + 1 + 1
    sdpa_bytes = sdpa_algorithmic_bytes(cfg, cap["cnt"])
    reps = 3
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    with torch.no_grad():
        ops.sparse_sdpa(cap["dims"], cap["q"], cap["k"], cap["v"], cap["sel"], cap["cnt"], cap["gate"], m.scale)
        torch.cuda.synchronize()
        s0.record()
        for _ in range(reps):
            ops.sparse_sdpa(cap["dims"], cap["q"], cap["k"], cap["v"], cap["sel"], cap["cnt"], cap["gate"],
                            m.scale)
        s1.record()
        torch.cuda.synchronize()
    sdpa_ms = s0.elapsed_time(s1) / reps
    pk, pk_kind = peaks()
    clocks = clk.summary()
    roofline = sdpa_roofline(cfg, cap["cnt"], sdpa_ms, sdpa_bytes, pk, pk_kind, clocks, dev,
                             args.workload, B, L, world)

    roofline_indexer = indexer_roofline(cap, cfg, pk)
    roofline_proj = proj_roofline(m, x, pk)
    x_mib = B * L * cfg.d_model * 2 / 2**20
    kv_mib = B * L * cfg.n_kv_heads * cfg.d_head * 2 / 2**20
    res = {
        "metric": METRIC if (args.workload == "prefill" and L == 131072) else PREFILL_METRIC,
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: x ~ N(0,1) seed 1, default-init weights seed 0",
        "config": {"workload": prefill_workload_name(B, L, k_min, k_max),
                   "batch": B, "seq_len": L,
                   "parallelism": f"query-sequence shards x{world}" +
                                  ((f" (zigzag, {ZIGZAG_FOLDS} folds)" if zigzag else " (contiguous)")
                                   if world > 1 else ""),
                   "l2": (f"inputs larger than L2 (x {x_mib:.0f} MiB, K/V {kv_mib:.0f} MiB each)"
                          if x_mib > 126 else f"x {x_mib:.0f} MiB: L2 not flushed between steps"),
                   "candidates": (f"{cap.get('survivor_pass')} survivors"
                                  if cap.get("candidate_path") == "survivors" else "exact top-k")},
        "e2e": e2e, "roofline": roofline, "roofline_indexer": roofline_indexer, "roofline_proj": roofline_proj,
        "gpu_launches": launches_per_step * args.steps,
        "stages_ms": stages, "clocks": clocks,
    }
    if shard_balance is not None:
        res["shards"] = shard_balance
    return res


# ---------------------------------------------------------------------------------------------
# decode workload: 64 sequences x 65,536 cached tokens, one new token each per step
# ---------------------------------------------------------------------------------------------
DECODE_SEQS = 64
DECODE_CACHED = 65536
DECODE_METRIC = "GSA layer decode tokens/sec, 64 seqs x 1 new token vs 65,536 cached (B200)"


def decode_step_bytes(cfg, n_seqs: int, n_keys: int, cnt: torch.Tensor) -> dict:
    """Bytes one decode step must move from HBM: the layer's weights (fused projection and
    o_proj, bf16), every cached indexer key (d_I bf16 per key), the selected K and V rows
    (Hk*D bf16 each) with their int32 indices, and the per-token vectors (x, q, gate, out)."""
    H, Hk, D, dI = cfg.n_heads, cfg.n_kv_heads, cfg.d_head, cfg.d_indexer
    n_cat = H * D + 3 * Hk * D + H * D + cfg.n_indexer_heads * dI + dI + cfg.n_indexer_heads
    weights = (n_cat + H * D) * cfg.d_model * 2
    ki = n_seqs * n_keys * dI * 2
    sum_k = float(cnt.double().sum().item())
    kv = sum_k * (2 * Hk * D * 2 + 4)
    vec = n_seqs * (2 * cfg.d_model + 3 * H * D) * 2
    return {"weights": weights, "indexer_keys": ki, "kv_rows": kv, "vectors": vec,
            "total": weights + ki + kv + vec}


def run_decode(args, world, rank):
    from gsa_b200 import GSAConfig, GatedSparseAttention, ops
    from gsa_b200.sharded import enable_sequence_sharding

    dev = torch.device("cuda", torch.cuda.current_device())
    n_cached = args.cached
    if DECODE_SEQS % world:
        raise SystemExit(f"{DECODE_SEQS} sequences do not divide over {world} ranks")
    B = DECODE_SEQS // world
    total_steps = args.warmup + 2 * args.steps + 2
    cfg = GSAConfig(**WORKLOAD, max_position_embeddings=n_cached + total_steps + 1)
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).eval().to(torch.bfloat16).to(dev)
    if world > 1:
        import torch.distributed as dist

        enable_sequence_sharding(m, dist.group.WORLD)
    # the cache: N(0,1) K, V and indexer keys (seed 2; this rank's sequences), room for every step
    cache = m.allocate_cache(B, n_cached + total_steps)
    g = torch.Generator(device=dev).manual_seed(2 + rank)
    st = cache.store
    for b in range(B):
        st.kv[b, :n_cached].normal_(generator=g)
        st.ki[b, :n_cached].normal_(generator=g)
    st.filled = n_cached
    cache = st.view(n_cached)
    gen = torch.Generator().manual_seed(1 + rank)
    x_host = torch.randn(total_steps, B, 1, cfg.d_model, generator=gen).to(torch.bfloat16).pin_memory()
    xs = x_host.to(dev)
    torch.cuda.synchronize()
    it = [0]

    def step(c, x=None):
        x = xs[it[0]] if x is None else x
        it[0] += 1
        with torch.no_grad():
            out, c, _ = m(x, past_key_value=c, use_cache=True)
        return out, c

    for _ in range(args.warmup):
        _, cache = step(cache)
    torch.cuda.synchronize()
    ops.check_device_error()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if world == 1 else int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            _, cache = step(cache)
        end.record()
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    value = DECODE_SEQS / (ms / 1e3)

    # end to end: each step's token copied from pinned host memory, its output read back
    out_host = torch.empty(B, 1, cfg.d_model, dtype=torch.bfloat16).pin_memory()
    barrier(world)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        xd = x_host[it[0]].to(dev, non_blocking=True)
        out, cache = step(cache, xd)
        out_host.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    e2e = {"value": DECODE_SEQS / (e2e_ms / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": out_host.numel() * 2 * world, "d2h_bytes_per_step": out_host.numel() * 2 * world,
           "ms_per_step": e2e_ms}

    # one more step with stage marks and captured selections; kernels timed alone
    cap, marks = {}, []

    def mark(name):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        marks.append((name, ev))

    n_keys = cache[0].shape[1] + 1
    with torch.no_grad():
        # the stage-by-stage path (the same kernels launched one by one from Python); one call
        # first so that its buffers are allocated before the marked call
        m._forward_impl(xs[it[0]], None, cache, False, False, capture={})
        torch.cuda.synchronize()
        e_start = torch.cuda.Event(enable_timing=True)
        e_start.record()
        m._forward_impl(xs[it[0]], None, cache, False, False, mark=mark, capture=cap)
    torch.cuda.synchronize()
    stages, prev = {}, e_start
    for name, ev in marks:
        stages[name] = round(prev.elapsed_time(ev), 4)
        prev = ev
    pk, pk_kind = peaks()
    nbytes = decode_step_bytes(cfg, B, n_keys, cap["cnt"])
    reps = 20

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    import ctypes as C
    from gsa_b200 import _lib

    qI, kI, w, shift = cap["qI"], cap["kI"], cap["w"], cap["shift"]
    ld = (n_keys + 3) // 4 * 4
    scratch = torch.empty(B * ld, device=dev, dtype=torch.float32)
    wv = w.reshape(-1, cfg.n_indexer_heads).float().contiguous()
    bias = cap["bias"].float().contiguous()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def indexer():
        _lib.call("gsa_indexer_scores", C.byref(cap["dims"]), ops.dtype_code(qI.dtype), B, 1, n_keys, n_keys - 1, 1,
                  0, C.c_void_p(qI.data_ptr()), qI.stride(1), qI.stride(0), C.c_void_p(kI.data_ptr()), kI.stride(1),
                  kI.stride(0), C.c_void_p(wv.data_ptr()), C.c_void_p(bias.data_ptr()), float(cap["idx_scale"]),
                  C.c_void_p(shift.data_ptr()), C.c_void_p(scratch.data_ptr()), ld, None, stream)

    def sdpa():
        ops.sparse_sdpa(cap["dims"], cap["q"], cap["k"], cap["v"], cap["sel"], cap["cnt"], cap["gate"], m.scale)

    with torch.no_grad():
        idx_ms = timed(indexer)
        sdpa_ms = timed(sdpa)
    hbm = pk["hbm_gbs"]

    def rl(name, b, t_ms):
        a = b / (t_ms / 1e3) / 1e9
        return {"kernel": name, "bound": "hbm", "achieved": round(a, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(a / hbm, 4), "peak_kind": pk_kind, "algorithmic_bytes": b, "kernel_ms": round(t_ms, 4)}

    roofline = rl("decode step (all kernels and GEMMs, device time per step)", nbytes["total"], ms)
    roofline["traffic"] = None
    roofline["bytes"] = nbytes
    parts = {"indexer": rl("gsa::dec::indexer_decode_kernel<8,1,4>", nbytes["indexer_keys"], idx_ms),
             "sdpa": rl("gsa::sdpa_tc_kernel<128,4>", nbytes["kv_rows"] + B * 3 * cfg.n_heads * cfg.d_head * 2,
                        sdpa_ms)}
    # our kernels per step (gsa_decode_attend): projection epilogue, decode indexer, survivor count +
    # write + exact fallback, variance and adaptive k (one kernel for one GPU; row variance + their
    # sum, then adaptive k, around the all-reduce of the sharded step), final selection, split SDPA
    # + merge
    var_launches = (1 if world == 1 else 3) if cfg.use_adaptive_k else 1
    launches_per_step = 1 + 1 + 3 + var_launches + 1 + 2
    return {
        "metric": DECODE_METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: cache K, V, k^I ~ N(0,1) seed 2, new tokens x ~ N(0,1) seed 1, default-init weights seed 0",
        "config": {"workload": f"GSA layer decode {DECODE_SEQS} seqs x 1 token vs {n_cached}+ cached "
                               "d4096 h32/8x128 idx8x64 k2048[256,4096] bf16",
                   "batch": DECODE_SEQS, "cached": n_cached, "parallelism": f"sequence shards x{world}",
                   "l2": "inputs larger than L2 (cache 17 GB)"},
        "e2e": e2e, "roofline": roofline, "roofline_kernels": parts, "mean_k": float(cap["cnt"].double().mean()),
        "gpu_launches": launches_per_step * args.steps,
        "stages_ms": stages, "stages_note": "one step launched stage by stage from Python (the timed steps are "
                                            "one native call between the two GEMMs)",
        "clocks": clk.summary(),
    }


# ---------------------------------------------------------------------------------------------
# training step: forward + backward of the layer
# ---------------------------------------------------------------------------------------------
TRAIN_METRIC = "GSA layer fwd+bwd tokens/sec (training step, B200)"


def sdpa_backward_bytes(cfg, cnt: torch.Tensor) -> float:
    """Bytes the SDPA backward must move: per selected key the K and V rows (bf16) read and the
    dK, dV rows (fp32) accumulated; per row q, O, dO read (bf16), dq written (fp32), lse."""
    Hk, H, D = cfg.n_kv_heads, cfg.n_heads, cfg.d_head
    sum_k = float(cnt.double().sum().item())
    return sum_k * (2 * Hk * D * 2 + 2 * Hk * D * 4 + 4) + cnt.numel() * (3 * H * D * 2 + H * D * 4 + H * 4)


def run_train(args, world, rank):
    from gsa_b200 import GSAConfig, GatedSparseAttention, ops

    dev = torch.device("cuda", torch.cuda.current_device())
    L = args.seq_len or 131072
    cfg = GSAConfig(**WORKLOAD, max_position_embeddings=max(131072, L))
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).to(torch.bfloat16).to(dev).train()
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(1, L, cfg.d_model, generator=gen).to(torch.bfloat16).to(dev).requires_grad_(True)
    dy = torch.randn(1, L, cfg.d_model, generator=gen).to(torch.bfloat16).to(dev)

    def step():
        m.zero_grad(set_to_none=True)
        x.grad = None
        out = m(x)[0]
        out.backward(dy)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.check_device_error()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    # forward alone (the training forward: the SDPA without its fused gate, log-sum-exp kept)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        m(x)[0]
    f1.record()
    torch.cuda.synchronize()
    fwd_ms = f0.elapsed_time(f1) / args.steps
    # the SDPA backward kernel alone on this step's selection
    saved = {}
    with torch.no_grad():
        m._forward_impl(x.detach(), None, None, False, False, train=saved)
        d_o = torch.randn_like(saved["O"])
        ops.sparse_sdpa_backward(saved["dims"], saved["q"], saved["k"], saved["v"], saved["sel"], saved["cnt"],
                                 saved["O"], d_o, saved["lse"], m.scale)
        torch.cuda.synchronize()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record()
        reps = 3
        for _ in range(reps):
            ops.sparse_sdpa_backward(saved["dims"], saved["q"], saved["k"], saved["v"], saved["sel"], saved["cnt"],
                                     saved["O"], d_o, saved["lse"], m.scale)
        b1.record()
        torch.cuda.synchronize()
    bwd_kernel_ms = b0.elapsed_time(b1) / reps
    pk, pk_kind = peaks()
    nbytes = sdpa_backward_bytes(cfg, saved["cnt"])
    achieved = nbytes / (bwd_kernel_ms / 1e3) / 1e9
    return {
        "metric": TRAIN_METRIC, "value": round(L / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: x, dy ~ N(0,1) seed 1, default-init weights seed 0",
        "config": {"workload": f"GSA layer fwd+bwd B=1 L={L} d4096 h32/8x128 idx8x64 k2048[256,4096] bf16",
                   "batch": 1, "seq_len": L, "parallelism": "single GPU"},
        "forward_ms": round(fwd_ms, 3), "backward_ms": round(ms - fwd_ms, 3),
        "roofline": {"kernel": "gsa::bwd::sdpa_bwd_kernel<bf16,4,4>", "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                     "peak_kind": pk_kind, "algorithmic_bytes": nbytes, "kernel_ms": round(bwd_kernel_ms, 3),
                     "traffic": None},
        "gpu_launches": None, "clocks": clk.summary(),
    }


# ---------------------------------------------------------------------------------------------
# decoder layer: RMSNorm + GSA + residual + RMSNorm + SwiGLU MLP + residual
# ---------------------------------------------------------------------------------------------
LAYER_METRIC = "GSA decoder layer fwd tokens/sec (RMSNorm, GSA, SwiGLU d_ffn 11008; B200)"


def run_layer(args, world, rank):
    from gsa_b200 import GSAConfig, GSADecoderLayer, ops

    dev = torch.device("cuda", torch.cuda.current_device())
    L = args.seq_len or 131072
    cfg = GSAConfig(**WORKLOAD, max_position_embeddings=max(131072, L))
    torch.manual_seed(0)
    m = GSADecoderLayer(cfg, 0).eval().to(torch.bfloat16).to(dev)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(1, L, cfg.d_model, generator=gen).to(torch.bfloat16).to(dev)

    def step():
        with torch.no_grad():
            return m(x)[0]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.check_device_error()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    # the attention alone on the normed input, for the split
    with torch.no_grad():
        normed = m.input_layernorm(x)
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(args.steps):
            m.self_attn(normed)
        a1.record()
        torch.cuda.synchronize()
    attn_ms = a0.elapsed_time(a1) / args.steps
    mlp_flops = 2.0 * L * cfg.d_model * cfg.d_ffn * 3
    return {
        "metric": LAYER_METRIC, "value": round(L / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: x ~ N(0,1) seed 1, default-init weights seed 0",
        "config": {"workload": f"GSA decoder layer fwd B=1 L={L} d4096 h32/8x128 idx8x64 k2048[256,4096] "
                               f"ffn{cfg.d_ffn} bf16", "batch": 1, "seq_len": L, "parallelism": "single GPU"},
        "attention_ms": round(attn_ms, 3), "rest_ms": round(ms - attn_ms, 3),
        "mlp_tflops": round(mlp_flops / ((ms - attn_ms) / 1e3) / 1e12, 1),
        "gpu_launches": None, "clocks": clk.summary(),
    }


# ---------------------------------------------------------------------------------------------
# CPU path of the reference algorithm (oracle restatement), sampled and extrapolated
# ---------------------------------------------------------------------------------------------
CPU_SAMPLE = dict(proj_rows=128, chunk_rows=16, n_chunks=4)
_WEIGHTS = {}


def _oracle_weights(O, oc, seed, dt):
    """The layer's weights from the oracle's restatement of the reference's init, built once per
    process (outside every timed sample)."""
    key = (seed, dt, oc.k_min, oc.k_max)
    if key not in _WEIGHTS:
        _WEIGHTS[key] = O.init_layer_weights(oc, seed, dtype=dt)
    return _WEIGHTS[key]


def cpu_reference_estimate(B: int, L: int, k_min: int, k_max: int, proj_rows: int, chunk_rows: int,
                           n_chunks: int, seed: int = 0):
    """Seconds for one layer forward over B sequences of L tokens on the host cores, estimated from
    samples timed with the oracle's restatement of the reference's torch ops (bf16, torch.no_grad,
    weights from the oracle's restatement of the reference's seeded init):
      * projections + G2 + RoPE + G1 logits + o_proj on ``proj_rows`` rows, scaled by B*L/rows;
      * indexer + variance for ``n_chunks`` chunks of ``chunk_rows`` queries at evenly spaced
        offsets, scaled by the causal (query, key) pair count of the B sequences;
      * top-k + sparse attention for the same chunks, scaled by B*L / sampled rows.
    Returns (seconds, description)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import torch.nn.functional as F

    import gsa_oracle as O

    torch.set_num_threads(len(os.sched_getaffinity(0)))
    oc = O.OracleConfig(**{**WORKLOAD, "k_min": k_min, "k_max": k_max}, d_head=128)
    dt = torch.bfloat16
    W = _oracle_weights(O, oc, seed, dt)
    cos_t, sin_t = (t.to(dt) for t in O.rope_cache(oc.d_head, max(proj_rows, 16), oc.rope_base, oc.rope_scaling))
    gen = torch.Generator().manual_seed(1)
    H, Hk, D = oc.n_heads, oc.n_kv_heads, oc.d_head
    with torch.no_grad():
        # 1. dense projections and gates, per row
        xs = torch.randn(1, proj_rows, oc.d_model, generator=gen).to(dt)
        pos = torch.arange(proj_rows).unsqueeze(0)
        t0 = time.perf_counter()
        q, k, v = O.project(W, oc, xs, pos, cos_t, sin_t)
        F.linear(xs, W["indexer.q_proj.weight"])
        F.linear(xs, W["indexer.k_proj.weight"])
        g = F.linear(xs, W["output_gate.gate_proj.weight"], W["output_gate.gate_proj.bias"])
        gated = q * O.gate_activation(g.view(1, proj_rows, H, D), "sigmoid")
        F.linear(gated.reshape(1, proj_rows, -1), W["o_proj.weight"])
        t_proj = (time.perf_counter() - t0) * B * L / proj_rows
        # 2./3. indexer, variance, top-k, sparse attention on sampled query chunks
        kI = torch.randn(1, L, oc.d_indexer, generator=gen).to(dt)
        K = torch.randn(1, L, Hk, D, generator=gen).to(dt)
        V = torch.randn(1, L, Hk, D, generator=gen).to(dt)
        t_idx = t_sel = 0.0
        pairs_sampled = 0
        rows_sampled = 0
        k_eff = min(oc.k_max, L)
        for c in range(n_chunks):
            t_pos = min(int((c + 0.5) * L / n_chunks), L - chunk_rows)
            n_keys = t_pos + chunk_rows
            xq = torch.randn(1, chunk_rows, oc.d_model, generator=gen).to(dt)
            t1 = time.perf_counter()
            q_idx = F.linear(xq, W["indexer.q_proj.weight"]).view(1, chunk_rows, oc.n_indexer_heads, oc.d_indexer)
            wts = torch.sigmoid(F.linear(xq, W["indexer.weight_proj.weight"], W["indexer.weight_proj.bias"]))
            sc = O.indexer_scores_from_proj(q_idx, kI[:, :n_keys], wts, W["indexer.bias"], "sigmoid", q_offset=t_pos)
            full = torch.full((1, chunk_rows, L), float("-inf"), dtype=sc.dtype)
            full[:, :, :n_keys] = sc
            var, valid = O.row_variance(full)
            t2 = time.perf_counter()
            kv = O.adaptive_k(var, valid, var.mean(), oc.k_base, oc.k_min, oc.k_max, 1.0)
            idx, msk = O.topk_select(full, k_eff, kv)
            qc = torch.randn(1, chunk_rows, H, D, generator=gen).to(dt)
            O.sparse_attention(qc, K, V, idx, msk, oc.n_heads // oc.n_kv_heads, 1.0 / math.sqrt(D))
            t3 = time.perf_counter()
            t_idx += t2 - t1
            t_sel += t3 - t2
            pairs_sampled += sum(t_pos + i + 1 for i in range(chunk_rows))
            rows_sampled += chunk_rows
        total_pairs = B * L * (L + 1) / 2
        est = t_proj + t_idx * total_pairs / pairs_sampled + t_sel * B * L / rows_sampled
    desc = (f"sampled + extrapolated: projections/gates/o_proj on {proj_rows} rows x {B}*L/{proj_rows}; "
            f"indexer+variance on {n_chunks} chunks of {chunk_rows} queries x causal pairs; "
            f"top-k+sparse attention on the same chunks x {B}*L/{rows_sampled}; weights from the oracle's init")
    return est, desc


def cpu_decode_estimate(n_cached: int, n_sample: int = 4, seed: int = 0):
    """Seconds for one step of the 64-sequence decode workload on the host cores, timed with the
    oracle's restatement of the reference's torch ops (bf16, torch.no_grad): the projections,
    gates and o_proj for all 64 new tokens; the indexer over every cached key, the variance,
    top-k and sparse attention for ``n_sample`` sequences, scaled by 64 / n_sample.
    Returns (seconds, description)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import torch.nn.functional as F

    import gsa_oracle as O

    torch.set_num_threads(len(os.sched_getaffinity(0)))
    cfg = O.OracleConfig(**WORKLOAD, d_head=128, max_position_embeddings=n_cached + 8)
    oc = cfg
    dt = torch.bfloat16
    W = _oracle_weights(O, oc, seed, dt)
    cos_t, sin_t = (t.to(dt) for t in O.rope_cache(oc.d_head, n_cached + 8, oc.rope_base, oc.rope_scaling))
    gen = torch.Generator().manual_seed(2)
    H, Hk, D, HI, dI = cfg.n_heads, cfg.n_kv_heads, cfg.d_head, cfg.n_indexer_heads, cfg.d_indexer
    S, n = n_sample, n_cached + 1
    with torch.no_grad():
        K = torch.randn(S, n, Hk, D, generator=gen).to(dt)
        V = torch.randn(S, n, Hk, D, generator=gen).to(dt)
        kI = torch.randn(S, n, dI, generator=gen).to(dt)
        x = torch.randn(DECODE_SEQS, 1, cfg.d_model, generator=gen).to(dt)
        pos = torch.full((DECODE_SEQS, 1), n_cached)
        t0 = time.perf_counter()
        q, k, v = O.project(W, oc, x, pos, cos_t, sin_t)
        q_idx = F.linear(x, W["indexer.q_proj.weight"]).view(DECODE_SEQS, 1, HI, dI)
        k_new = F.linear(x, W["indexer.k_proj.weight"])
        wts = torch.sigmoid(F.linear(x, W["indexer.weight_proj.weight"], W["indexer.weight_proj.bias"]))
        g1 = O.gate_activation(F.linear(x, W["output_gate.gate_proj.weight"],
                                        W["output_gate.gate_proj.bias"]).view(DECODE_SEQS, 1, H, D), "sigmoid")
        F.linear((q * g1).reshape(DECODE_SEQS, 1, -1), W["o_proj.weight"])
        t_dense = time.perf_counter() - t0
        t1 = time.perf_counter()
        K[:, -1:], V[:, -1:], kI[:, -1:] = k[:S], v[:S], k_new[:S]
        sc = O.indexer_scores_from_proj(q_idx[:S], kI, wts[:S], W["indexer.bias"], "sigmoid", q_offset=n_cached)
        var, valid = O.row_variance(sc)
        k_t = O.adaptive_k(var, valid, var.mean(), cfg.k_base, cfg.k_min, cfg.k_max, 1.0)
        idx, msk = O.topk_select(sc, min(cfg.k_max, n), k_t)
        O.sparse_attention(q[:S], K, V, idx, msk, H // Hk, 1.0 / math.sqrt(D))
        t_seq = (time.perf_counter() - t1) * DECODE_SEQS / S
    desc = (f"projections/gates/o_proj for all {DECODE_SEQS} tokens; indexer over {n} keys, variance, "
            f"top-k and sparse attention for {S} sequences x {DECODE_SEQS}/{S}")
    return t_dense + t_seq, desc


def run_reference(args, world, rank):
    """Reference arm: the reference algorithm's CPU path, timed on this box's host cores."""
    if args.workload == "decode":
        samples, desc = [], ""
        for i in range(args.warmup + args.steps):
            sec, desc = cpu_decode_estimate(args.cached)
            if i >= args.warmup:
                samples.append(sec)
        sec = statistics.median(samples)
        v = DECODE_SEQS / sec
        cores = len(os.sched_getaffinity(0))
        return {"metric": DECODE_METRIC, "value": round(v, 3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 1),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic: cache ~ N(0,1), x ~ N(0,1), default-init weights seed 0",
                "config": {"workload": f"GSA layer decode {DECODE_SEQS} seqs x 1 token vs {args.cached} cached "
                                       "d4096 h32/8x128 idx8x64 k2048[256,4096] bf16",
                           "batch": DECODE_SEQS, "cached": args.cached, "parallelism": "host CPU"},
                "impl": "reference",
                "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                                 "sample": desc},
                "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    B, L, k_min, k_max = prefill_shape(args)
    samples = []
    desc = ""
    for i in range(args.warmup + args.steps):
        est, desc = cpu_reference_estimate(B, L, k_min, k_max, seed=0, **CPU_SAMPLE)
        if i >= args.warmup:
            samples.append(est)
    sec = statistics.median(samples)
    v = B * L / sec
    cores = len(os.sched_getaffinity(0))
    return {"metric": METRIC if (args.workload == "prefill" and L == 131072) else PREFILL_METRIC,
            "value": round(v, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: x ~ N(0,1), default-init weights seed 0",
            "config": {"workload": prefill_workload_name(B, L, k_min, k_max),
                       "batch": B, "seq_len": L, "parallelism": "host CPU"},
            "impl": "reference",
            "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": desc},
            "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_selection_overlap(args):
    """Key sharing between nearby rows' selections (one 1-GPU forward of the prefill workload): for
    sampled row blocks across the sequence, |S_t & S_(t+j)| / |S_t| for j = 1..16, and the union of
    the selections of 8 and 16 consecutive rows against the sum of their sizes.  Prints one JSON
    line (a measurement, not a benchmark)."""
    from gsa_b200 import GSAConfig, GatedSparseAttention

    torch.cuda.set_device(0)
    B, L, k_min, k_max = prefill_shape(args)
    cfg = GSAConfig(**{**WORKLOAD, "k_min": k_min, "k_max": k_max}, max_position_embeddings=max(131072, L))
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).eval().to(torch.bfloat16).cuda()
    x = torch.randn(B, L, cfg.d_model, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).cuda()
    cap = {}
    with torch.no_grad():
        m._forward_impl(x, None, None, False, False, capture=cap)
    sel, cnt = cap["sel"], cap["cnt"].long()
    del cap, x
    torch.cuda.empty_cache()
    starts = [int(f * L) // 16 * 16 for f in (0.125, 0.25, 0.375, 0.5, 0.625, 0.75, 0.875)]
    starts = [t for t in starts if t + 32 <= L]
    lag = {j: [] for j in range(1, 17)}
    union8, union16 = [], []
    for t0 in starts:
        rows = torch.arange(t0, t0 + 32, device="cuda")
        mask = torch.zeros(32, L, dtype=torch.bool, device="cuda")
        for i, r in enumerate(rows.tolist()):
            mask[i, sel[r, :cnt[r]].long()] = True
        sizes = mask.sum(-1).double()
        for j in range(1, 17):
            inter = (mask[:16] & mask[j:16 + j]).sum(-1).double()
            lag[j].append(float((inter / sizes[:16]).mean()))
        for blk, out in ((8, union8), (16, union16)):
            for b0 in range(0, 32, blk):
                u = mask[b0:b0 + blk].any(0).sum().double()
                out.append(float(u / sizes[b0:b0 + blk].sum()))
    res = {"workload": prefill_workload_name(B, L, k_min, k_max), "row_blocks": starts,
           "mean_k": float(cnt.double().mean()),
           "shared_fraction_at_lag": {j: round(statistics.mean(v), 4) for j, v in lag.items()},
           "union_over_sum_8_rows": round(statistics.mean(union8), 4),
           "union_over_sum_16_rows": round(statistics.mean(union16), 4),
           "note": "shared_fraction_at_lag[j] = mean |S_t & S_(t+j)| / |S_t| over 16 rows t of each block; "
                   "union_over_sum = |S_t u ... u S_(t+n-1)| / sum |S_i| (1.0: no key shared)"}
    emit(res)


def run_launch_list(args):
    """N untimed forwards of the 1-GPU workload at --seq-len (or N decode steps against
    --cached tokens), for kernel profilers."""
    from gsa_b200 import GSAConfig, GatedSparseAttention, ops

    torch.cuda.set_device(0)
    if args.workload == "decode":
        cfg = GSAConfig(**WORKLOAD, max_position_embeddings=args.cached + args.launch_list + 1)
        torch.manual_seed(0)
        m = GatedSparseAttention(cfg).eval().to(torch.bfloat16).cuda()
        cache = m.allocate_cache(DECODE_SEQS, args.cached + args.launch_list)
        st = cache.store
        g = torch.Generator(device="cuda").manual_seed(2)
        st.kv[:, :args.cached].normal_(generator=g)
        st.ki[:, :args.cached].normal_(generator=g)
        st.filled = args.cached
        cache = st.view(args.cached)
        x = torch.randn(DECODE_SEQS, 1, cfg.d_model, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
        x = x.cuda()
        with torch.no_grad():
            for _ in range(args.launch_list):
                _, cache, _ = m(x, past_key_value=cache, use_cache=True)
        torch.cuda.synchronize()
        ops.check_device_error()
        log(f"launch list: {args.launch_list} decode steps against {args.cached} cached tokens done")
        return
    B, L, k_min, k_max = prefill_shape(args)
    cfg = GSAConfig(**{**WORKLOAD, "k_min": k_min, "k_max": k_max}, max_position_embeddings=max(131072, L))
    torch.manual_seed(0)
    m = GatedSparseAttention(cfg).eval().to(torch.bfloat16).cuda()
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(B, L, cfg.d_model, generator=gen).to(torch.bfloat16).cuda()
    with torch.no_grad():
        if args.sdpa_replay:
            # one forward keeps the SDPA's inputs; the forward's other buffers are released, and the
            # SDPA alone runs --sdpa-replay more times (a capture of the last launches holds only
            # q, gate, K/V, the selection and the output on the device)
            cap = {}
            m._forward_impl(x, None, None, False, False, capture=cap)
            keep = {k: cap[k] for k in ("dims", "q", "k", "v", "sel", "cnt", "gate")}
            del cap, x
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
            for _ in range(args.sdpa_replay):
                ops.sparse_sdpa(keep["dims"], keep["q"], keep["k"], keep["v"], keep["sel"], keep["cnt"],
                                keep["gate"], m.scale)
            torch.cuda.synchronize()
            ops.check_device_error()
            log(f"sdpa replay: {args.sdpa_replay} launches after one forward at B={B} L={L}; "
                f"{torch.cuda.memory_allocated() / 2**30:.2f} GiB held")
            return
        for _ in range(args.launch_list):
            m(x)
    torch.cuda.synchronize()
    ops.check_device_error()
    log(f"launch list: {args.launch_list} forwards at L={L} done")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seq-len", type=int, default=None,
                    help="tokens per sequence (prefill default: the workload's; train/layer: 131072)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--launch-list", type=int, default=0, metavar="N",
                    help="run N untimed forwards and exit (a short command for profilers)")
    ap.add_argument("--selection-overlap", action="store_true",
                    help="measure key sharing between nearby rows' selections (prefill workloads) and exit")
    ap.add_argument("--sdpa-replay", type=int, default=0, metavar="N",
                    help="with --launch-list: after one forward, run the sparse SDPA alone N times and exit")
    ap.add_argument("--workload", default="prefill", choices=["prefill", "c2", "c3", "decode", "train", "layer"],
                    help="prefill: one 131072-token sequence; c2: two 8192-token sequences; c3: one 32768-token "
                         "sequence with k in [512, 4096]; decode: 64 sequences x 1 token vs 65,536 cached; "
                         "train: forward + backward of one --seq-len sequence; layer: a whole decoder layer")
    ap.add_argument("--cached", type=int, default=DECODE_CACHED, help="decode: cached tokens per sequence")
    args = ap.parse_args()
    quiet_stdout()
    if args.selection_overlap:
        return run_selection_overlap(args)
    if args.launch_list:
        return run_launch_list(args)
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        res = run_reference(args, world, rank)
        res["n_gpus"] = world
        emit(res)
        return

    world, rank, local = dist_setup(args.gpus)
    try:
        if args.workload in ("train", "layer"):
            res = (run_train if args.workload == "train" else run_layer)(args, world, rank)
            if rank == 0:
                emit(res)
            return
        if args.workload == "decode":
            res = run_decode(args, world, rank)
            if rank == 0 and world == 1 and not args.no_cpu_baseline:
                sec, desc = cpu_decode_estimate(args.cached)
                res["cpu_baseline"] = {"value": round(DECODE_SEQS / sec, 3), "unit": "tokens/s",
                                       "cores": len(os.sched_getaffinity(0)), "kind": "port", "sample": desc}
            if rank == 0:
                emit(res)
            return
        res = run_ours(args, world, rank)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            # the reference arm's estimate, the median of three samples
            B, L, k_min, k_max = prefill_shape(args)
            ests = [cpu_reference_estimate(B, L, k_min, k_max, seed=0, **CPU_SAMPLE) for _ in range(3)]
            est, desc = statistics.median(e for e, _ in ests), ests[0][1]
            res["cpu_baseline"] = {"value": round(B * L / est, 3), "unit": "tokens/s",
                                   "cores": len(os.sched_getaffinity(0)), "kind": "port",
                                   "sample": desc + "; median of 3"}
        if rank == 0:
            emit(res)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
