"""The reference arm of bench.py on the host (no GPU): the JSON line it prints
and its behaviour under several ranks (rank 0 alone measures and prints; the
other ranks exit 0 without work)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None, *args):
    env = dict(os.environ)
    env.update(extra_env or {})
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
           "--workload", "gemm_ffn_up", "--steps", "1", "--warmup", "0", *args]
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)


def _lines(out):
    return [json.loads(s) for s in out.splitlines() if s.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    r = _run()
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1
    d = lines[0]
    for key in ("metric", "value", "unit", "impl", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["warmup"] >= 3  # the contract's minimum, whatever was asked
    assert d["steps"] == 1 and d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"].startswith("gemm_ffn_up")
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_runs_on_rank_zero_only():
    other = _run({"RANK": "1", "WORLD_SIZE": "2"}, "--gpus", "2")
    assert other.returncode == 0, other.stderr[-2000:]
    assert _lines(other.stdout) == []
    first = _run({"RANK": "0", "WORLD_SIZE": "2"}, "--gpus", "2")
    assert first.returncode == 0, first.stderr[-2000:]
    assert len(_lines(first.stdout)) == 1
