"""The parts of bench.py that need no GPU: the timed CPU baseline (the
oracle on host threads, also the `--impl reference` arm) reports the keys the
benchmark line carries, on a tiny sample of the benchmark workload."""

from __future__ import annotations

import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import bench  # noqa: E402


def test_cpu_baseline_keys_and_rate():
    res = bench.cpu_oracle_rate(total_envs_hint=4, warmup=0, steps=1, threads=2)
    assert set(res) >= {"value", "unit", "cores", "kind", "cpu_model", "sample"}
    assert res["unit"] == bench.UNIT and res["kind"] == "port" and res["cores"] == 2
    assert res["value"] > 0
    assert "4 envs x 1 env-steps" in res["sample"]
    json.dumps(res)  # the line is JSON


def test_cpu_model_is_a_string():
    assert isinstance(bench._cpu_model(), str) and bench._cpu_model()
