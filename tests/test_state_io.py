"""PyBoy .state files: the parser and writer against the reference's own
state_io.py (golden vectors from tests/golden/make_state_fixtures.py)."""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

from gbxcule_b200 import state_io as sio
from tests.conftest import GOLDEN

GOLD = json.loads((GOLDEN / "state_io.json").read_text())["cases"]
BLOBS = np.load(GOLDEN / "state_io.npz")


def _sha(b: bytes) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def fields(state) -> dict:
    return {k: _sha(v) if isinstance(v, (bytes, bytearray)) else int(v) for k, v in vars(state).items()}


@pytest.mark.parametrize("version", [12, 13, 14, 15])
def test_parse_matches_reference_on_every_layout(version):
    case = GOLD[f"synthetic_v{version}"]
    data = BLOBS[f"synthetic_v{version}"].tobytes()
    ram = case["cart_ram_bytes"]
    assert fields(sio.parse_pyboy_state(data, expected_cart_ram_size=ram)) == case["loaded_hint"]
    assert fields(sio.parse_pyboy_state(data)) == case["loaded_nohint"]


@pytest.mark.parametrize("name", ["cfg2", "cfg4"])
def test_reference_saved_file_parses_and_rewrites_identically(name, tmp_path):
    case = GOLD[name]
    data = BLOBS[f"saved_{name}"].tobytes()
    assert _sha(data) == case["file_sha256"]
    st = sio.parse_pyboy_state(data, expected_cart_ram_size=case["cart_ram_bytes"])
    assert fields(st) == case["loaded"]
    assert sio.write_pyboy_state(st) == data  # the version-9 writer is byte-identical
    p = tmp_path / "x.state"
    sio.save_pyboy_state(st, p)
    assert fields(sio.load_pyboy_state(p, expected_cart_ram_size=case["cart_ram_bytes"])) == case["loaded"]


def test_errors_like_the_reference():
    data = bytearray(BLOBS["saved_cfg2"].tobytes())
    bad = bytes([8]) + bytes(data[1:])
    with pytest.raises(ValueError, match="Unsupported state version 8"):
        sio.parse_pyboy_state(bad)
    cgb = bytes(data[:4]) + b"\x01" + bytes(data[5:])
    with pytest.raises(ValueError, match="CGB mode not supported"):
        sio.parse_pyboy_state(cgb)
    with pytest.raises(ValueError, match="vram must be 8192 bytes"):
        st = sio.parse_pyboy_state(bytes(data))
        st.vram = b"\x00"
        sio.write_pyboy_state(st)
