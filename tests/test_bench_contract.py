"""The bench's reference arm on the CPU: one JSON line with the contract's keys.

``bench.py --impl reference`` times the CPU restatement of the funnel on the
host cores; the driver runs it beside the GPU arm and compares the two lines.
These tests run it on a small layer and check the line's shape, and that
ranks other than 0 of a multi-rank launch print nothing and exit 0.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
ARGS = ["--impl", "reference", "--steps", "2", "--warmup", "3", "--context", "16384", "--nprobe", "128"]


def _bench(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *ARGS], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    r = _bench({"WORLD_SIZE": "1", "RANK": "0", "LOCAL_RANK": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1
    assert d["steps"] == 2 and d["warmup"] == 3
    assert d["higher_is_better"] is False and d["unit"] == "µs/layer"
    assert d["value"] > 0 and d["ms_per_step"] == pytest.approx(d["value"] / 1e3)
    assert d["config"]["context"] == 16384 and d["config"]["nprobe"] == 128
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    r = _bench({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [x for x in r.stdout.splitlines() if x.startswith("{")]
