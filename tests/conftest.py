"""Shared fixtures. Tests that need a B200 are marked ``gpu``."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def golden():
    return json.loads((GOLDEN / "fixtures.json").read_text())["cases"]


@pytest.fixture(scope="session")
def micro_roms():
    with np.load(GOLDEN / "micro_roms.npz") as z:
        return {k: z[k].tobytes() for k in z.files}


def case_rom(case: dict, micro: dict) -> bytes:
    from gbxcule_b200 import roms

    if case["rom"]["kind"] == "config":
        return roms.CONFIG_ROMS[case["rom"]["id"]]()
    if case["rom"]["kind"] == "isa_probe":
        from tests import isa_probe

        return isa_probe.rom_image()
    return micro[case["rom"]["id"]]


def case_setup_state(case: dict, rom: bytes) -> dict | None:
    """Per-env start state a golden case writes after reset (None: reset alone)."""
    if case.get("setup") == "isa_probe":
        from tests import isa_probe

        return isa_probe.initial_state(rom)
    return None
