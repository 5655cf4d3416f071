"""Pin the CPU oracle to the reference: replay every golden case.

The digests in tests/golden/fixtures.json were produced by running the
reference's own backend and kernel source (tests/golden/ref_harness.py) on the
same ROMs, boot stub and actions; the oracle must reproduce every per-step
state digest, render digest and restore digest bit for bit.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from gbxcule_b200 import roms
from gbxcule_b200 import state as st
from oracle import OracleEnvs
from tests.conftest import case_rom, case_setup_state


def _sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def _cases():
    import json
    from tests.conftest import GOLDEN

    return json.loads((GOLDEN / "fixtures.json").read_text())["cases"]


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_oracle_matches_reference(case, micro_roms, monkeypatch):
    rom = case_rom(case, micro_roms)
    assert _sha(rom) == case["rom"]["sha256"], "ROM generator output changed"
    for k, v in case.get("env", {}).items():  # debug traps, read at construction
        monkeypatch.setenv(k, v)
    o = OracleEnvs(rom, roms.boot_stub(), case["num_envs"], stage=case["stage"])
    assert st.digest(o.state()) == case["reset_digest"]
    init = case_setup_state(case, rom)
    if init is not None:
        for name, arr in init.items():
            o.s[name][:] = np.asarray(arr).reshape(o.s[name].shape)
        assert st.digest(o.state()) == case["setup_digest"]
    trace = case["trace"]
    warm = case.get("warmup", 0)
    for rec in trace[:warm]:
        o.step(np.array(rec["actions"], dtype=np.int32), case["frames"], case["release"])
        assert st.digest(o.state()) == rec["digest"]
    snap = None
    if "restore" in case:
        rs = case["restore"]
        snap = o.snapshot(rs["snapshot_env"])
        o.restore(snap, np.ones(case["num_envs"], dtype=np.uint8))
        assert st.digest(o.state()) == rs["after_full_restore"]
    for k, rec in enumerate(trace[warm:]):
        o.step(np.array(rec["actions"], dtype=np.int32), case["frames"], case["release"])
        assert st.digest(o.state()) == rec["digest"], f"step {k}"
        if "frame_bg" in rec:
            assert _sha(o.render_bg_env0().tobytes()) == rec["frame_bg"], f"env-0 frame step {k}"
        if "render_packed" in rec:
            assert _sha(o.render_packed().tobytes()) == rec["render_packed"], f"packed render step {k}"
            assert _sha(o.render_shades().tobytes()) == rec["render_shades"], f"shade render step {k}"
        if "mask" in rec:
            o.restore(snap, np.array(rec["mask"], dtype=np.uint8))
            assert st.digest(o.state()) == rec["after_restore"], f"restore step {k}"
