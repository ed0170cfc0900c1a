"""bench.py's reference arm on the host: the one JSON line it prints carries
the metric, unit and configuration of the CUDA arm, a cpu_baseline that
describes the same run, and an e2e block with no host<->device bytes; under a
multi-rank launch only rank 0 runs and prints it. (The CUDA arm needs a GPU;
its line is checked where it runs.)"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ARGS = ["--impl", "reference", "--steps", "1", "--warmup", "1", "--image-size", "256",
        "--batch", "1"]


def run_bench(extra_env=None):
    env = dict(os.environ)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *ARGS], cwd=ROOT,
                          env=env, capture_output=True, text=True, timeout=600)


@pytest.fixture(scope="module")
def line():
    r = run_bench({"RANK": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_line_carries_the_contract_keys(line):
    for k in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
              "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["impl"] == "reference"
    assert line["metric"] == "encoder images/s" and line["unit"] == "images/s"
    assert line["higher_is_better"] is True
    assert line["value"] > 0
    assert abs(line["ms_per_step"] - 1e3 / line["value"]) < 1e-6 * line["ms_per_step"]
    assert line["config"]["image_size"] == 256 and line["config"]["global_batch"] == 1
    assert "workload" in line["config"]


def test_reference_cpu_baseline_describes_this_run(line):
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["unit"] == line["unit"]
    assert cb["kind"] in ("port", "reference")
    assert cb["cores"] >= 1 and cb["sample"]


def test_reference_e2e_moves_no_bytes(line):
    e = line["e2e"]
    assert e["value"] == line["value"] and e["unit"] == line["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_other_ranks_exit_quietly():
    r = run_bench({"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [l for l in r.stdout.splitlines() if l.startswith("{")]
