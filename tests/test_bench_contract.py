"""bench.py's driver contract, the parts that run without a GPU.

* ``--impl reference`` prints one JSON line with the contract's keys, an ``impl`` of
  "reference", a ``cpu_baseline`` describing the run and an ``e2e`` with no copies;
* under torchrun only rank 0 of the reference arm works and prints, the other ranks
  exit 0 without output;
* the roofline's ``traffic`` comes from the committed ncu summary of the workload.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def _bench(*args, env=None):
    full_env = dict(os.environ)
    full_env.update(env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=600, env=full_env, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    proc = _bench("--impl", "reference", "--steps", "2", "--warmup", "1", "--workload", "b1_h4_s512_noncausal")
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [line for line in proc.stdout.splitlines() if line.strip()]
    assert len(lines) == 1, proc.stdout
    line = json.loads(lines[0])
    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and line["unit"] == "TFLOPS" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 2 and line["warmup"] == 1
    assert line["cpu_baseline"]["value"] == line["value"] and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert "workload" in line["config"]


def test_reference_arm_other_ranks_exit_quietly():
    proc = _bench("--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1",
                  "--workload", "b1_h4_s512_noncausal", env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert proc.stdout.strip() == ""


def test_traffic_comes_from_the_committed_profile_summaries():
    sys.path.insert(0, str(ROOT))
    import importlib

    bench = importlib.import_module("bench")
    for workload in ("b4_h16_s4096_noncausal", "b2_h16_s8192_causal"):
        traffic = bench.profiled_traffic(workload)
        assert traffic is not None and 1e8 < traffic < 1e9, (workload, traffic)
    assert bench.profiled_traffic("no_such_workload") is None
