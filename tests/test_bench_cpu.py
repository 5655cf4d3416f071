"""The parts of bench.py that need no GPU: the reference arm's timer (the
oracle on host threads) on a tiny sample, the roofline arithmetic, and the
integer-issue constants against the committed ncu summaries they come from."""

from __future__ import annotations

import json
import re
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO))

import bench  # noqa: E402


@pytest.mark.parametrize("cfg", [2, 5])
def test_reference_rate_on_a_tiny_sample(cfg):
    value, setup_s, what = bench.reference_rate(cfg, threads=2, m=2, warmup=1, steps=1, warm_steps=1)
    assert value > 0 and setup_s >= 0
    assert ("restores" in what) == (cfg == 5)


def test_step_bytes_terms():
    b = bench.step_bytes(5, 1000.0, 0.05)
    want = (bench.ACTION_BYTES + 2 * bench.STATE_BYTES + bench.OBS_VEC_BYTES + 1000.0 + bench.R_OBS
            + bench.R_SRC + 0.05 * bench.RESTORE_BYTES[5])
    assert b == pytest.approx(want)
    assert bench.step_bytes(2, 0.0, 0.0) < b


def test_roofline_names_the_larger_fraction(monkeypatch):
    monkeypatch.setitem(bench.WARP_INSTR_PER_EMULATED_INSTR, "config5:uniform", (10.0, "x"))
    r = bench.roofline("config5:uniform", 5, 1000, kernel_ms=100.0, emu_instr_per_launch=1e9,
                       ram_ops_per_env_step=5e4, sm_count=148, sm_mhz=2000.0, restore_rate=0.05)
    issue = 10.0 * 1e9 / 0.1 / (148 * 4 * 2000e6)
    assert r["issue"]["frac"] == pytest.approx(issue)
    assert r["bound"] == ("integer-issue" if issue > r["hbm"]["frac"] else "hbm")
    assert r["frac"] == pytest.approx(max(issue, r["hbm"]["frac"]))
    json.dumps(r)
    # a shape without a committed capture has no issue roof
    r2 = bench.roofline("config5:switch", 5, 1000, kernel_ms=100.0, emu_instr_per_launch=1e9,
                        ram_ops_per_env_step=5e4, sm_count=148, sm_mhz=2000.0, restore_rate=0.05)
    assert r2["issue"] is None and r2["bound"] == "hbm"


def _profile_ratio(path: Path) -> float:
    """The 'warp instructions per emulated instruction' row of a profile summary."""
    m = re.search(r"\|\s*warp instructions per emulated instruction\s*\|\s*([0-9.]+)", path.read_text())
    assert m, f"{path} has no 'warp instructions per emulated instruction' row"
    return float(m.group(1))


@pytest.mark.parametrize("workload", sorted(bench.WARP_INSTR_PER_EMULATED_INSTR))
def test_issue_constants_match_the_profiles(workload):
    value, src = bench.WARP_INSTR_PER_EMULATED_INSTR[workload]
    if value is None:
        pytest.skip(f"{workload}: no capture for this build yet")
    assert _profile_ratio(REPO / src) == pytest.approx(value, rel=0.01)


def test_cpu_model_is_a_string():
    assert isinstance(bench._cpu_model(), str) and bench._cpu_model()
