"""The benchmark's output contract, checked on the host: ``bench.py --impl reference`` (the
reference algorithm's CPU path, timed on the host cores) prints exactly one JSON line with the
keys the result consumer reads, and under a multi-rank launch only rank 0 prints."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(extra_env=None, *args):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--seq-len", "2048",
                           "--steps", "1", *args], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    p = _run(None, "--warmup", "0")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, p.stdout
    r = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in r, key
    assert r["impl"] == "reference" and r["n_gpus"] == 1 and r["steps"] == 1
    assert r["warmup"] >= 3                                  # at least three warm-up steps, whatever is asked
    assert r["value"] > 0 and r["unit"] == "tokens/s" and r["higher_is_better"] is True
    assert r["config"]["seq_len"] == 2048 and r["config"]["batch"] == 1
    cb = r["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] == r["value"]
    e2e = r["e2e"]
    assert e2e["value"] == r["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_exit_quietly():
    p = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""


def test_reference_arm_takes_the_batch_of_two_workload():
    """The two-sequence workload (B=2): the arm's config and throughput count both sequences."""
    p = _run(None, "--warmup", "0", "--workload", "c2")
    assert p.returncode == 0, p.stderr[-2000:]
    r = json.loads(p.stdout.strip())
    assert r["config"]["batch"] == 2 and r["config"]["seq_len"] == 2048
    assert "B=2 L=2048" in r["config"]["workload"] and "k2048[256,4096]" in r["config"]["workload"]
    assert abs(r["value"] - 2 * 2048 / (r["ms_per_step"] / 1e3)) <= 1e-3 * r["value"] + 1e-3
