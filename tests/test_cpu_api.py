"""CPU-only checks: the C-ABI library loads and exports every declared symbol,
argument validation happens before any device call, and the pure-Python
pieces (header parse, generators, action projection) behave."""

from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest

from gbxcule_b200 import _lib as L
from gbxcule_b200 import cartridge as cart
from gbxcule_b200 import roms
from tests.conftest import REPO


def _declared():
    text = (REPO / "include" / "gbx.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int32_t|const char\*)\s+(gbx_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    names = _declared()
    assert len(names) >= 20
    for name in names:
        assert hasattr(lib, name), name
    assert lib.gbx_abi_version() == L.ABI_VERSION == 5


def test_create_validates_before_touching_a_device():
    lib = L.lib()
    h = ctypes.c_void_p()
    cfg = L.Config(4, 0, 1, 0, 0)
    rom = bytearray(roms.config1_rom())
    boot = roms.boot_stub()
    rom[0x147] = 0x05  # MBC2: unsupported by the reference too
    rc = lib.gbx_create(ctypes.byref(cfg), bytes(rom), len(rom), boot, 256, ctypes.byref(h))
    assert rc == L.GBX_ERR_INVALID and b"Unsupported cartridge type" in lib.gbx_last_error()
    rc = lib.gbx_create(ctypes.byref(cfg), roms.config1_rom(), 0x8000, boot, 255, ctypes.byref(h))
    assert rc == L.GBX_ERR_INVALID and b"256 bytes" in lib.gbx_last_error()
    rc = lib.gbx_create(ctypes.byref(cfg), roms.config1_rom()[:0x4000], 0x4000, boot, 256, ctypes.byref(h))
    assert rc == L.GBX_ERR_INVALID and b"smaller than header" in lib.gbx_last_error()
    with pytest.raises(ValueError):
        L.check(L.GBX_ERR_RANGE)
    with pytest.raises(RuntimeError):
        L.check(L.GBX_ERR_STATE)


def test_null_handles_are_rejected():
    lib = L.lib()
    assert lib.gbx_reset(None, None) == L.GBX_ERR_INVALID
    assert lib.gbx_step(None, None, 1, 1, None) == L.GBX_ERR_INVALID
    assert lib.gbx_destroy(None) == L.GBX_OK
    assert lib.gbx_snapshot_destroy(None) == L.GBX_OK
    assert lib.gbx_set_envs_per_warp(None, 4) == L.GBX_ERR_INVALID
    assert lib.gbx_set_dispatch(None, 2) == L.GBX_ERR_INVALID
    assert lib.gbx_render_packed_scaled(None, None, 0, None, 0, None) == L.GBX_ERR_INVALID


def test_generators_are_deterministic_with_valid_headers():
    for k, fn in roms.CONFIG_ROMS.items():
        a, b = fn(), fn()
        assert a == b, k
        x = 0
        for byte in a[0x134:0x14D]:
            x = (x - byte - 1) & 0xFF
        assert a[0x14D] == x
        assert (sum(a[:0x14E]) + sum(a[0x150:])) & 0xFFFF == (a[0x14E] << 8 | a[0x14F])
        spec = cart.parse_cartridge_header(a)
        assert spec.rom_byte_length == len(a)
    assert cart.parse_cartridge_header(roms.config4_rom()).mbc_kind == cart.MBC_KIND_MBC3
    assert len(roms.boot_stub()) == 256 and roms.boot_stub()[0xFE:] == bytes([0xE0, 0x50])


def test_header_parse_errors_like_the_reference():
    rom = bytearray(roms.config1_rom())
    with pytest.raises(ValueError, match="too small"):
        cart.parse_cartridge_header(bytes(rom[:0x100]))
    rom[0x148] = 0x09
    with pytest.raises(ValueError, match="ROM size code"):
        cart.parse_cartridge_header(bytes(rom))
    rom[0x148] = 0x00
    rom[0x149] = 0x01  # 2 KiB: not a whole 8 KiB bank
    with pytest.raises(ValueError, match="Invalid RAM byte length"):
        cart.parse_cartridge_header(bytes(rom))


def test_bernoulli_projection():
    rng = np.random.default_rng(0)
    a = roms.bernoulli_actions(rng, 20000, 0.3)
    assert a.min() >= 0 and a.max() <= 7
    # P(no press among the 7 mapped buttons) with SELECT ignored
    assert abs((a == 0).mean() - 0.7 ** 7) < 0.02
    assert abs((a == 1).mean() - 0.3) < 0.02
