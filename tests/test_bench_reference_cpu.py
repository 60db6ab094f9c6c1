"""The bench's reference arm (``bench.py --impl reference``) on a tiny workload: one JSON
line with the driver's keys, the reference's metric and unit, a ``cpu_baseline`` that
describes the run and an ``e2e`` record with no host<->device bytes. It times the oracle
port of the reference's PyTorch path on the host cores, so it runs without a GPU."""

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--N", "64", "--layers", "1",
           "--steps", "1", "--warmup", "0", "--cpu-rows", "16"]
    env = dict(os.environ, WORLD_SIZE="1", RANK="0", LOCAL_RANK="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["higher_is_better"] is True and d["value"] > 0
    assert d["metric"].startswith("pair-stack layers*N^2/sec") and d["unit"] == "layers*N^2/s"
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] == "port"
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_is_silent_on_other_ranks():
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--N", "64", "--layers", "1",
           "--steps", "1", "--warmup", "0", "--cpu-rows", "16", "--gpus", "2"]
    env = dict(os.environ, WORLD_SIZE="2", RANK="1", LOCAL_RANK="1")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
