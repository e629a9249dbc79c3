"""bench.py's reference arm, run on the CPU: the JSON line the driver parses.

`bench.py --impl reference` times the oracle's C decode on the host cores and
prints one line on rank 0 carrying the arm's metric, unit, direction,
`impl`, a `cpu_baseline` that describes the run and an `e2e` with no
host-device copies; any other rank exits 0 without work or output.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import PROJECT, REPO


def _run(extra_env):
    env = dict(os.environ)
    env.update(extra_env)
    env["PYTHONPATH"] = os.pathsep.join([str(PROJECT), str(REPO), env.get("PYTHONPATH", "")])
    cmd = [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
           "--warmup", "3"]
    return subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600, cwd=REPO)


def test_reference_arm_line():
    r = _run({})
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["metric"] == "paged decode-attn HBM GB/s" and line["unit"] == "GB/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    assert line["warmup"] >= 3 and line["steps"] == 1
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    assert line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_do_nothing():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
