"""
bench.py's output contract, on the CPU: the reference arm (the CPU oracle port
of the reference's attention, timed on the host cores) prints one JSON line
with the keys the driver reads, for the same metric, unit and workload as the
B200 arm; and the B200 arm fails loudly (non-zero exit) on a machine without a
GPU instead of falling back to anything.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def run(*args, timeout=600):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    import bench

    r = run("--impl", "reference", "--steps", "3", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == bench.UNIT == "tok/s"
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert (d["n_gpus"], d["steps"], d["warmup"]) == (1, 3, 3)
    assert d["higher_is_better"] is True and d["scaling"] == "weak" and d["vs_baseline"] is None
    assert d["data"] == "synthetic" and d["config"]["workload"] == bench.WORKLOAD
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"] and cb["kind"] == "port"
    assert cb["cores"] >= 1 and cb["sample"]
    e = d["e2e"]
    assert e == {"value": e["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert e["value"] == pytest.approx(d["value"], rel=1e-3)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_b200_arm_fails_loudly_without_a_gpu():
    r = run("--steps", "3", "--warmup", "3", timeout=300)
    assert r.returncode != 0
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")], "no result line without a GPU"
