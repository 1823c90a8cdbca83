"""bench.py's reference arm on the host cores: one JSON line with the keys the bench contract
names, the same metric/unit/config as the GPU arm's default workload, and nothing printed by a
rank other than 0 (those exit 0 without work).  Runs without a GPU."""
from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e")


def run_bench(*args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    p = subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    return [ln for ln in p.stdout.splitlines() if ln.startswith("{")]


def test_reference_arm_line():
    lines = run_bench("--impl", "reference", "--steps", "2", "--warmup", "1")
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in KEYS:
        assert k in d, k
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["higher_is_better"] is True
    assert d["unit"] == "GB/s" and d["value"] > 0 and d["steps"] >= 1
    assert d["config"]["workload"].startswith("config0") and (d["config"]["n"], d["config"]["k"]) == (9728, 2560)
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    lines = run_bench("--impl", "reference", "--gpus", "2", "--steps", "2", "--warmup", "1",
                      env_extra={"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert lines == []


def test_reference_arm_config_keys_match_ours():
    """both arms print the same config keys and warm-up for the default workload"""
    sys.path.insert(0, ROOT)
    import bench
    lines = run_bench("--impl", "reference", "--steps", "2", "--warmup", "5")
    d = json.loads(lines[0])
    assert set(d["config"]) == set(bench.gemv_config(1))
    assert d["warmup"] == 5
    st = d["cpu_baseline"]["single_thread"]
    if d["cpu_baseline"]["kind"] == "reference":
        assert st["cores"] == 1 and st["value"] > 0
