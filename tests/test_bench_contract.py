"""bench.py's JSON contract, checked on CPU through its reference arm (the C
restatement of the reference's CPU path on the tiny model): one JSON line
with the contract's keys, at least 3 warm-up steps, and the reference arm's
cpu_baseline and zero-copy e2e."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(tmp_path, *extra):
    env = dict(os.environ, CXM_MODEL_DIR=str(tmp_path))
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "tiny",
                        "--steps", "2", "--prompt", "16", *extra], capture_output=True, text=True, env=env,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_prints_one_contract_line(tmp_path):
    d = _run(tmp_path, "--warmup", "1")
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference"
    assert d["warmup"] >= 3          # the contract's floor, whatever was asked
    assert d["value"] > 0 and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["config"]["workload"].startswith("tiny")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    # timed on the reference's x86 kernels, each format's kernel named
    assert "x86 AVX2 path" in cb["sample"] and "Q4_K: " in cb["sample"] and "Q6_K: " in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
