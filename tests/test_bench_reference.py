"""bench.py's reference arm on the host cores: the JSON line it prints and
its multi-rank behaviour (rank 0 runs and prints, the other ranks exit 0
without work). No GPU: the arm times the oracle's CPU algorithm."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _run(extra_env, *args):
    env = dict(os.environ, OMP_NUM_THREADS="2", **extra_env)
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--n", "256", "--steps", "1", "--warmup", "3", *args],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    return out.stdout.strip()


def test_reference_line_single_gpu():
    d = json.loads(_run({"RANK": "0"}))
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["unit"] == "iter/s" and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    assert d["config"]["N"] == 256 and d["config"]["M"] == 256
    assert d["warmup"] >= 3 and d["steps"] == 1


def test_reference_line_matches_the_weak_row_sharded_workload():
    d = json.loads(_run({"RANK": "0"}, "--gpus", "4"))
    assert d["n_gpus"] == 4 and d["scaling"] == "weak"
    assert d["config"]["N"] == 4 * 256 and d["config"]["M"] == 256
    assert "block-iterations per second" in d["config"]["workload"]
    assert "block-iterations per second" in d["cpu_baseline"]["sample"]


def test_reference_arm_other_ranks_exit_quietly():
    assert _run({"RANK": "1"}, "--gpus", "2") == ""
