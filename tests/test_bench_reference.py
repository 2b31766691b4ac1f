"""CPU: bench.py's reference arm (the reference's CPU algorithm through the oracle port on the
host cores) prints one JSON line with the contract's keys, alone and under torchrun with two ranks
(rank 0 alone runs and prints; the other rank exits 0 without work)."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT

KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _lines(out: str):
    return [json.loads(l) for l in out.splitlines() if l.startswith("{")]


def _check(line, n_gpus):
    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and line["n_gpus"] == n_gpus and line["steps"] == 1
    assert line["value"] > 0 and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_one_process():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1
    _check(lines[0], 1)
    assert lines[0]["config"]["workload"] == "c3-mine" and lines[0]["unit"] == "int8 TOPS"


def test_reference_arm_two_ranks():
    env = dict(os.environ, MASTER_ADDR="127.0.0.1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", "29533", "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
           "--warmup", "1"]
    try:
        r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    except subprocess.TimeoutExpired:
        pytest.fail("torchrun reference arm timed out")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1
    _check(lines[0], 2)
