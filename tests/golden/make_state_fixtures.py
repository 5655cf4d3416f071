"""Golden vectors for PyBoy ``.state`` I/O, produced by the reference's own
``src/gbxcule/core/state_io.py`` running under ``ref_harness``.

TEST INFRASTRUCTURE. Run only where the reference tree is available:

    python tests/golden/make_state_fixtures.py --reference <path-to-gbxcule>

Writes ``state_io.json`` (digests) and ``state_io.npz`` (the file bytes):

* ``saved_<cfg>``: the reference backend stepped from reset with seeded
  actions, then ``state_from_warp_backend`` + ``save_pyboy_state`` of one
  env: the file bytes, the digest of the source batch, and the fields the
  reference loader parses back;
* ``applied_<cfg>``: that state applied to env 0 of a fresh reference
  backend (``apply_state_to_warp_backend``), its full-state digest, then two
  more steps;
* ``synthetic_v<N>``: files in the version-12..15 layouts, built here from a
  seed (the reference writes only version 9), and the fields the reference
  loader parses with and without the cartridge-RAM size hint.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))

from gbxcule_b200 import roms  # noqa: E402
from gbxcule_b200 import state as st  # noqa: E402

STATE_CASES = [  # (name, config, envs, steps, source env, action seed)
    ("cfg2", 2, 2, 3, 1, 41),
    ("cfg4", 4, 2, 4, 1, 42),
]


def _sha(b: bytes) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def fields_digest(state) -> dict:
    """JSON-able view of a PyBoyState: ints as is, byte fields by sha256."""
    out = {}
    for k, v in vars(state).items():
        out[k] = _sha(v) if isinstance(v, (bytes, bytearray)) else int(v)
    return out


def synthetic_file(version: int, seed: int, cart_ram_size: int, samples: int = 5) -> bytes:
    """A state file in the given version's layout with seeded contents."""
    rng = np.random.default_rng(seed)
    rb = lambda n: rng.integers(0, 256, n, dtype=np.uint8).tobytes()  # noqa: E731
    u8 = lambda v: bytes([v & 0xFF])  # noqa: E731
    u16 = lambda v: struct.pack("<H", v & 0xFFFF)  # noqa: E731
    u64 = lambda v: struct.pack("<Q", v)  # noqa: E731
    b = bytearray()
    b += u8(version) + u8(1) + u8(0) + u8(0) + u8(0)
    b += rb(6) + u16(0x1234) + u16(0xDFF0) + u16(0x0150) + u8(1) + u8(0) + u8(0) + u8(0x1F) + u8(0) + u8(0x03)
    if version >= 12:
        b += u64(123456789)
    b += rb(8192) + rb(160) + rb(11) + u8(0) + u8(0)
    if version >= 13:
        b += u64(777)
    b += u64(456 * 100 + 17) + u64(456 * 101) + u8(2) + rb(720)
    # sound
    if version <= 12:
        b += rb(138)
    else:
        if version >= 14:
            b += u64(3) + u64(samples) + u64(0) + rb((samples + 1) * 2) + u8(0) + rb(8 * 7) + u8(1) + u8(0) + rb(8)
        else:
            b += rb(16)
        tone = 2 + 3 + 2 + 1 + 1 + 8 * 6
        b += rb(tone + 3 + 8 + 1 + 8) + rb(tone) + rb(16 + 1 + 1 + 1 + 2 + 1 + 1 + 8 * 5) + rb(8 + 1 + 8 * 7)
    b += bytes(144 * 160 * 5 if version >= 13 else 144 * 160 * 4 - 138)
    b += rb(8192) + rb(96) + rb(76) + rb(127) + rb(52)
    b += rb(2) + u16(0xBEEF) + u16(0x0042) + rb(2)
    if version >= 12:
        b += u64(99)
    if version >= 13:
        b += u64(98)
    b += u16(0x1F) + u8(2) + u8(1) + u8(0) + rb(cart_ram_size)
    b += u8(0x0E) + u8(0x0D)
    if version >= 15:
        b += u8(0x41) + u8(0x81) + u8(1) + u8(0) + rb(32)
    return bytes(b)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    import ref_harness as rh

    tmp = Path(tempfile.mkdtemp(prefix="gbxstate_"))
    boot = tmp / "boot.bin"
    boot.write_bytes(roms.boot_stub())
    ref = rh.load_reference(args.reference, boot)
    sio = __import__("gbxcule.core.state_io", fromlist=["x"])
    blobs: dict[str, np.ndarray] = {}
    cases: dict[str, dict] = {}
    for name, cfg, n, steps, env, seed in STATE_CASES:
        rom = roms.CONFIG_ROMS[cfg]()
        rom_path = tmp / f"{name}.gb"
        rom_path.write_bytes(rom)
        be = ref.backend(str(rom_path), num_envs=n, frames_per_step=24, release_after_frames=8)
        be.reset()
        rng = np.random.default_rng(seed)
        acts = []
        for _ in range(steps):
            a = roms.uniform_actions(rng, n, 9)
            acts.append(a.tolist())
            ref.launch_step(be, a)
        src_digest = st.digest({k: getattr(be, v).numpy() for k, v in st.REF_ATTR.items()})
        state = sio.state_from_warp_backend(be, env)
        path = tmp / f"{name}.state"
        sio.save_pyboy_state(state, path)
        data = path.read_bytes()
        ram = int(be._ram_byte_length)
        loaded = sio.load_pyboy_state(path, expected_cart_ram_size=ram)
        blobs[f"saved_{name}"] = np.frombuffer(data, dtype=np.uint8)
        be2 = ref.backend(str(rom_path), num_envs=n, frames_per_step=24, release_after_frames=8)
        be2.reset()
        sio.apply_state_to_warp_backend(loaded, be2, 0)
        applied = st.digest({k: getattr(be2, v).numpy() for k, v in st.REF_ATTR.items()})
        after = []
        arng = np.random.default_rng(seed + 100)
        for _ in range(2):
            a = roms.uniform_actions(arng, n, 9)
            ref.launch_step(be2, a)
            after.append({"actions": a.tolist(),
                          "digest": st.digest({k: getattr(be2, v).numpy() for k, v in st.REF_ATTR.items()})})
        cases[name] = {"config": cfg, "num_envs": n, "env": env, "actions": acts, "source_digest": src_digest,
                       "file_sha256": _sha(data), "file_bytes": len(data), "cart_ram_bytes": ram,
                       "loaded": fields_digest(loaded), "applied_digest": applied, "after": after}
        print(f"{name}: {len(data)} bytes")
    for version in (12, 13, 14, 15):
        ram = 8192 if version % 2 else 0
        data = synthetic_file(version, 500 + version, ram)
        path = tmp / f"v{version}.state"
        path.write_bytes(data)
        blobs[f"synthetic_v{version}"] = np.frombuffer(data, dtype=np.uint8)
        cases[f"synthetic_v{version}"] = {
            "cart_ram_bytes": ram,
            "loaded_hint": fields_digest(sio.load_pyboy_state(path, expected_cart_ram_size=ram)),
            "loaded_nohint": fields_digest(sio.load_pyboy_state(path)),
        }
        print(f"synthetic v{version}: {len(data)} bytes")
    np.savez_compressed(HERE / "state_io.npz", **blobs)
    (HERE / "state_io.json").write_text(json.dumps({
        "about": "PyBoy .state golden vectors from the reference's own state_io.py under ref_harness "
                 "(make_state_fixtures.py)", "cases": cases}, indent=1))


if __name__ == "__main__":
    main()
