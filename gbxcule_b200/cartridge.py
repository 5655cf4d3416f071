"""Cartridge header parsing and the per-env ``cart_state`` layout.

Mirrors ``src/gbxcule/core/cartridge.py`` of bkase/gbxcule: the same supported
cart types (ROM only, MBC1 family, MBC3 family), size codes, bank arithmetic
and the int32[20] per-env cart-state record (``:56-76``), so savestates and
snapshots line up field for field with the reference backend.
"""

from __future__ import annotations

from dataclasses import dataclass

CART_ROM_BANK_SIZE = 0x4000
CART_RAM_BANK_SIZE = 0x2000
BOOTROM_SIZE = 0x100

MBC_KIND_ROM_ONLY = 0
MBC_KIND_MBC1 = 1
MBC_KIND_MBC3 = 2

CART_STATE_STRIDE = 20
CART_STATE_FIELDS = (
    "mbc_kind", "ram_enable", "rom_bank_lo", "rom_bank_hi", "ram_bank", "bank_mode",
    "bootrom_enabled", "rtc_select", "rtc_latch", "rtc_seconds", "rtc_minutes",
    "rtc_hours", "rtc_days_low", "rtc_days_high", "rtc_last_cycle",
    "rtc_latched_seconds", "rtc_latched_minutes", "rtc_latched_hours",
    "rtc_latched_days_low", "rtc_latched_days_high",
)
CS = {name: k for k, name in enumerate(CART_STATE_FIELDS)}

_MBC1 = {0x01, 0x02, 0x03}
_MBC3 = {0x0F, 0x10, 0x11, 0x12, 0x13}
_SUPPORTED = {0x00} | _MBC1 | _MBC3

ROM_SIZE_MAP = {
    0x00: 32 * 1024, 0x01: 64 * 1024, 0x02: 128 * 1024, 0x03: 256 * 1024,
    0x04: 512 * 1024, 0x05: 1024 * 1024, 0x06: 2 * 1024 * 1024,
    0x07: 4 * 1024 * 1024, 0x08: 8 * 1024 * 1024,
    0x52: int(1.1 * 1024 * 1024), 0x53: int(1.2 * 1024 * 1024), 0x54: int(1.5 * 1024 * 1024),
}
RAM_SIZE_MAP = {0x00: 0, 0x01: 2 * 1024, 0x02: 8 * 1024, 0x03: 32 * 1024,
                0x04: 128 * 1024, 0x05: 64 * 1024}


@dataclass(frozen=True)
class CartridgeSpec:
    cart_type: int
    rom_byte_length: int
    rom_bank_count: int
    rom_bank_mask: int          # -1 when the bank count is not a power of two
    ram_byte_length: int
    ram_bank_count: int
    mbc_kind: int


def _pow2(v: int) -> bool:
    return v > 0 and (v & (v - 1)) == 0


def parse_cartridge_header(rom: bytes) -> CartridgeSpec:
    """Parse 0x147-0x149; raises ``ValueError`` like the reference parser."""
    if len(rom) < 0x150:
        raise ValueError(f"ROM too small for header: {len(rom)} bytes")
    ct = rom[0x147]
    if ct not in _SUPPORTED:
        raise ValueError(f"Unsupported cartridge type: 0x{ct:02X}")
    rc, ac = rom[0x148], rom[0x149]
    if rc not in ROM_SIZE_MAP:
        raise ValueError(f"Unsupported ROM size code: 0x{rc:02X}")
    if ac not in RAM_SIZE_MAP:
        raise ValueError(f"Unsupported RAM size code: 0x{ac:02X}")
    rom_bytes, ram_bytes = ROM_SIZE_MAP[rc], RAM_SIZE_MAP[ac]
    if rom_bytes % CART_ROM_BANK_SIZE:
        raise ValueError(f"Invalid ROM byte length: {rom_bytes}")
    if ram_bytes % CART_RAM_BANK_SIZE:
        raise ValueError(f"Invalid RAM byte length: {ram_bytes}")
    banks = rom_bytes // CART_ROM_BANK_SIZE
    kind = MBC_KIND_MBC1 if ct in _MBC1 else MBC_KIND_MBC3 if ct in _MBC3 else MBC_KIND_ROM_ONLY
    return CartridgeSpec(ct, rom_bytes, banks, banks - 1 if _pow2(banks) else -1,
                         ram_bytes, ram_bytes // CART_RAM_BANK_SIZE, kind)


def load_rom(rom: bytes) -> tuple[bytes, CartridgeSpec]:
    """Validate and trim a ROM image to the size its header advertises."""
    spec = parse_cartridge_header(rom)
    if len(rom) < spec.rom_byte_length:
        raise ValueError(f"ROM smaller than header advertises: {len(rom)} < {spec.rom_byte_length}")
    return bytes(rom[: spec.rom_byte_length]), spec
