"""bench.py --impl reference on CPU: the CPU restatement of the reference
backend timed on the host cores prints one JSON line with the same metric and
config as the B200 arm; under torchrun only rank 0 runs it and the other
ranks exit 0 without work.  The synthetic model goes to a temporary folder."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(tmp_path, extra_env=None):
    env = dict(os.environ, SLM_BENCH_DIR=str(tmp_path))
    env.update(extra_env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                           "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line(tmp_path):
    r = _run(tmp_path)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "decode tok/s, R=4, 4096 ctx full" and d["unit"] == "tok/s"
    assert d["higher_is_better"] is True and d["value"] > 0 and d["warmup"] >= 3
    assert d["config"]["workload"].startswith("C2 decode") and d["config"]["loops"] == 4
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_work(tmp_path):
    r = _run(tmp_path, {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
    assert not any(tmp_path.iterdir())  # no synthetic model written either
