"""PyBoy ``.state`` files (DMG): read versions 9-15, write version 9.

Same behaviour as the reference's ``src/gbxcule/core/state_io.py`` (the
parser ``_load_pyboy_state_from_file`` :275-550, the v9 writer :565-660 and
the conversions to and from a backend, ``state_from_warp_backend`` :662-836
and ``apply_state_to_warp_backend`` :839-1154), so a state saved by either
loads into the other. The conversions go through the backend's host state
export/import (``export_state`` / ``import_state``); nothing here runs on the
step path.

File layout (all integers little-endian), in order:
header (version, bootrom_enabled, key1, double_speed, cgb), CPU (A F B C D E,
HL, SP, PC, IME, halted, stopped, IE, interrupt_queued, IF, [v12+ cycles u64]),
LCD (VRAM 8192, OAM 160, LCDC BGP OBP0 OBP1 STAT LY LYC SCY SCX WY WX, cgb,
double speed, [v13+ last_cycles u64], clock u64, clock_target u64,
next_stat_mode, scanline params 720), sound (138 bytes before v13; field
layout in v13; v14+ sized from the file when the cartridge RAM size is
known), renderer (92022 or 115200 bytes before v13, chosen by which leaves a
valid cartridge RAM size; 115200 from v13), RAM (WRAM 8192, FEA0-FEFF 96,
IO FF00-FF4B 76, HRAM 127, FF4C-FF7F 52), timer (DIV, TIMA, DIV counter u16,
TIMA counter u16, TMA, TAC, [v12+ u64], [v13+ u64]), cartridge (ROM bank u16,
RAM bank, RAM enabled, memory model, RAM bytes up to the tail), tail
(joypad directional, joypad standard, [v15+ serial: SB, SC, two flags, 4 x u64]).
"""

from __future__ import annotations

import io
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Any, BinaryIO

import numpy as np

VERSION_MIN, VERSION_MAX, VERSION_SAVE = 9, 15, 9
VRAM, OAM, WRAM, HRAM, IO_PORTS, RAM_FEA0, RAM_FF4C = 8192, 160, 8192, 127, 76, 96, 52
SCANLINE_PARAMS = 720
SOUND_V9 = 138
RENDERER_OLD = 144 * 160 * 4 - 138  # 92022: PyBoy v9-v12 files
RENDERER = 144 * 160 * 5            # 115200: v13+ and files written here
CART_RAM_SIZES = (0, 2048, 8192, 32768, 131072)
CYCLES_PER_LINE = 456
SCREEN_H = 144


@dataclass
class PyBoyState:
    """One DMG state, field for field as the reference's ``PyBoyState``."""

    version: int
    bootrom_enabled: int
    a: int
    f: int
    b: int
    c: int
    d: int
    e: int
    h: int
    l_reg: int
    sp: int
    pc: int
    ime: int
    halted: int
    stopped: int
    ie: int
    interrupt_queued: int
    if_reg: int
    cpu_cycles: int
    vram: bytes
    oam: bytes
    lcdc: int
    stat: int
    ly: int
    lyc: int
    scy: int
    scx: int
    wy: int
    wx: int
    bgp: int
    obp0: int
    obp1: int
    lcd_clock: int
    lcd_clock_target: int
    next_stat_mode: int
    scanline_params: bytes
    wram: bytes
    hram: bytes
    io_ports: bytes
    non_io_ram0: bytes
    non_io_ram1: bytes
    div: int
    tima: int
    tma: int
    tac: int
    div_counter: int
    tima_counter: int
    rombank: int
    rambank: int
    rambank_enabled: int
    memorymodel: int
    cart_ram: bytes
    joypad_directional: int
    joypad_standard: int
    serial_sb: int
    serial_sc: int


class _Reader:
    def __init__(self, f: BinaryIO) -> None:
        self.f = f

    def u8(self) -> int:
        b = self.f.read(1)
        if len(b) != 1:
            raise EOFError("Unexpected end of file")
        return b[0]

    def u16(self) -> int:
        b = self.f.read(2)
        if len(b) != 2:
            raise EOFError("Unexpected end of file")
        return struct.unpack("<H", b)[0]

    def u64(self) -> int:
        b = self.f.read(8)
        if len(b) != 8:
            raise EOFError("Unexpected end of file")
        return struct.unpack("<Q", b)[0]

    def raw(self, n: int) -> bytes:
        return self.f.read(n)

    def skip(self, n: int) -> None:
        self.f.read(n)

    def size(self) -> int:
        here = self.f.tell()
        end = self.f.seek(0, 2)
        self.f.seek(here)
        return end


# sound channel records (PyBoy's save order), skipped
def _skip_tone(r: _Reader) -> None:
    r.skip(2 + 3 + 2 + 1 + 1 + 8 * 6)


def _skip_sweep(r: _Reader) -> None:
    _skip_tone(r)
    r.skip(3 + 8 + 1 + 8)


def _skip_wave(r: _Reader) -> None:
    r.skip(16 + 1 + 1 + 1 + 2 + 1 + 1 + 8 * 5)


def _skip_noise(r: _Reader) -> None:
    r.skip(8 + 1 + 8 * 7)


def _timer_bytes(version: int) -> int:
    return 8 + (8 if version >= 12 else 0) + (8 if version >= 13 else 0)


def _skip_sound(r: _Reader, version: int, cart_ram_size: int | None) -> None:
    if version == 13:
        r.skip(16)  # last_cycles, cycles
    elif version >= 14:
        if cart_ram_size is not None:
            after = (RENDERER + WRAM + RAM_FEA0 + IO_PORTS + HRAM + RAM_FF4C + _timer_bytes(version) + 5
                     + cart_ram_size + 2 + (36 if version >= 15 else 0))
            n = r.size() - r.f.tell() - after + (1 if version >= 15 else 0)
            if n < 0:
                raise ValueError(f"State file too small for sound section: {n} bytes")
            r.skip(n)
            return
        r.skip(8)                 # audiobuffer head
        samples = r.u64()         # samples per frame
        r.skip(8 + (samples + 1) * 2 + 1 + 8 + 8 + 8 + 8 + 8 + 8 + 8 + 1 + 1 + 8)
    else:
        r.skip(SOUND_V9)
        return
    _skip_sweep(r)
    _skip_tone(r)
    _skip_wave(r)
    _skip_noise(r)


def _renderer_bytes(r: _Reader, version: int) -> int:
    if version >= 13:
        return RENDERER
    remaining = r.size() - r.f.tell()
    after = WRAM + RAM_FEA0 + IO_PORTS + HRAM + RAM_FF4C + _timer_bytes(version) + 5 + 2
    old_ram = remaining - RENDERER_OLD - after
    new_ram = remaining - RENDERER - after
    old_ok, new_ok = old_ram in CART_RAM_SIZES, new_ram in CART_RAM_SIZES
    if new_ok and not old_ok:
        return RENDERER
    if old_ok:
        return RENDERER_OLD
    return RENDERER_OLD if old_ram >= 0 else RENDERER


def read_pyboy_state(f: BinaryIO, *, expected_cart_ram_size: int | None = None) -> PyBoyState:
    """Parse a state from an open binary file (versions 9-15, DMG only)."""
    r = _Reader(f)
    version = r.u8()
    if not VERSION_MIN <= version <= VERSION_MAX:
        raise ValueError(f"Unsupported state version {version}, expected {VERSION_MIN}-{VERSION_MAX}")
    bootrom = r.u8()
    r.skip(2)  # key1, double speed
    if r.u8() != 0:
        raise ValueError("CGB mode not supported, only DMG")
    a, flags, b, c, d, e = (r.u8() for _ in range(6))
    hl, sp, pc = r.u16(), r.u16(), r.u16()
    ime, halted, stopped, ie, queued, if_reg = (r.u8() for _ in range(6))
    cpu_cycles = r.u64() if version >= 12 else 0
    vram, oam = r.raw(VRAM), r.raw(OAM)
    lcdc, bgp, obp0, obp1, stat, ly, lyc, scy, scx, wy, wx = (r.u8() for _ in range(11))
    r.skip(2)  # cgb, double speed
    if version >= 13:
        r.skip(8)  # last_cycles
    lcd_clock, lcd_target = r.u64(), r.u64()
    next_mode = r.u8()
    scan = r.raw(SCANLINE_PARAMS)
    _skip_sound(r, version, expected_cart_ram_size)
    r.skip(_renderer_bytes(r, version))
    wram, fea0, io_ports, hram, ff4c = r.raw(WRAM), r.raw(RAM_FEA0), r.raw(IO_PORTS), r.raw(HRAM), r.raw(RAM_FF4C)
    div, tima = r.u8(), r.u8()
    div_counter, tima_counter = r.u16(), r.u16()
    tma, tac = r.u8(), r.u8()
    r.skip(_timer_bytes(version) - 8)
    rombank, rambank, ram_en, model = r.u16(), r.u8(), r.u8(), r.u8()
    serial_bytes = 36 if version >= 15 else 0
    start = r.f.tell()
    cart_n = r.size() - 2 - serial_bytes - start
    if cart_n < 0:
        raise ValueError(f"State file too small for cart RAM: {cart_n} bytes remaining")
    cart_ram = r.raw(cart_n) if cart_n else b""
    if len(cart_ram) != cart_n:
        raise EOFError("Unexpected end of file while reading cart RAM")
    r.f.seek(-(serial_bytes + 2), 2)
    joy_dir, joy_std = r.u8(), r.u8()
    if version >= 15:
        sb, sc = r.u8(), r.u8()
    else:
        sb, sc = io_ports[0x01], io_ports[0x02]
    return PyBoyState(
        version=version, bootrom_enabled=bootrom, a=a, f=flags, b=b, c=c, d=d, e=e,
        h=(hl >> 8) & 0xFF, l_reg=hl & 0xFF, sp=sp, pc=pc, ime=ime, halted=halted, stopped=stopped,
        ie=ie, interrupt_queued=queued, if_reg=if_reg, cpu_cycles=cpu_cycles, vram=vram, oam=oam,
        lcdc=lcdc, stat=stat, ly=ly, lyc=lyc, scy=scy, scx=scx, wy=wy, wx=wx, bgp=bgp, obp0=obp0,
        obp1=obp1, lcd_clock=lcd_clock, lcd_clock_target=lcd_target, next_stat_mode=next_mode,
        scanline_params=scan, wram=wram, hram=hram, io_ports=io_ports, non_io_ram0=fea0,
        non_io_ram1=ff4c, div=div, tima=tima, tma=tma, tac=tac, div_counter=div_counter,
        tima_counter=tima_counter, rombank=rombank, rambank=rambank, rambank_enabled=ram_en,
        memorymodel=model, cart_ram=cart_ram, joypad_directional=joy_dir, joypad_standard=joy_std,
        serial_sb=sb, serial_sc=sc)


def load_pyboy_state(path: str | Path, *, expected_cart_ram_size: int | None = None) -> PyBoyState:
    """Load a ``.state`` file (reference ``load_pyboy_state``, state_io.py:253-272)."""
    with open(Path(path), "rb") as f:
        return read_pyboy_state(f, expected_cart_ram_size=expected_cart_ram_size)


def write_pyboy_state(state: PyBoyState) -> bytes:
    """The version-9 file bytes of ``state`` (sound and renderer sections zero)."""
    out = bytearray()
    u8 = lambda v: out.append(int(v) & 0xFF)  # noqa: E731
    u16 = lambda v: out.extend(struct.pack("<H", int(v) & 0xFFFF))  # noqa: E731
    u64 = lambda v: out.extend(struct.pack("<Q", int(v) & 0xFFFFFFFFFFFFFFFF))  # noqa: E731

    def blob(b: bytes, n: int, what: str) -> None:
        if len(b) != n:
            raise ValueError(f"{what} must be {n} bytes, got {len(b)}")
        out.extend(b)

    for v in (VERSION_SAVE, state.bootrom_enabled & 1, 0, 0, 0):
        u8(v)
    for v in (state.a, state.f, state.b, state.c, state.d, state.e):
        u8(v)
    u16((state.h << 8) | state.l_reg)
    u16(state.sp)
    u16(state.pc)
    for v in (state.ime, state.halted, state.stopped, state.ie, state.interrupt_queued, state.if_reg):
        u8(v)
    blob(state.vram, VRAM, "vram")
    blob(state.oam, OAM, "oam")
    for v in (state.lcdc, state.bgp, state.obp0, state.obp1, state.stat, state.ly, state.lyc, state.scy,
              state.scx, state.wy, state.wx, 0, 0):
        u8(v)
    u64(state.lcd_clock)
    u64(state.lcd_clock_target)
    u8(state.next_stat_mode)
    blob(state.scanline_params, SCANLINE_PARAMS, "scanline_params")
    out.extend(bytes(SOUND_V9 + RENDERER))
    blob(state.wram, WRAM, "wram")
    blob(state.non_io_ram0, RAM_FEA0, "non_io_ram0")
    blob(state.io_ports, IO_PORTS, "io_ports")
    blob(state.hram, HRAM, "hram")
    blob(state.non_io_ram1, RAM_FF4C, "non_io_ram1")
    u8(state.div)
    u8(state.tima)
    u16(state.div_counter)
    u16(state.tima_counter)
    u8(state.tma)
    u8(state.tac)
    u16(state.rombank)
    u8(state.rambank)
    u8(state.rambank_enabled)
    u8(state.memorymodel)
    out.extend(state.cart_ram or b"")
    u8(state.joypad_directional)
    u8(state.joypad_standard)
    return bytes(out)


def save_pyboy_state(state: PyBoyState, path: str | Path) -> None:
    """Write ``state`` as a version-9 file (reference ``save_pyboy_state``, :553-562)."""
    Path(path).write_bytes(write_pyboy_state(state))


def parse_pyboy_state(data: bytes, *, expected_cart_ram_size: int | None = None) -> PyBoyState:
    """Parse state file bytes already in memory."""
    return read_pyboy_state(io.BytesIO(data), expected_cart_ram_size=expected_cart_ram_size)


# ---------------------------------------------------------------------------
# Backend conversions
# ---------------------------------------------------------------------------

def _mode_of(ly: int, scan: int) -> int:
    return 1 if ly >= SCREEN_H else 2 if scan < 80 else 3 if scan < 252 else 0


def state_from_backend(backend: Any, env_idx: int = 0) -> PyBoyState:
    """Env ``env_idx`` of a backend as a ``PyBoyState`` (state_io.py:662-836)."""
    if not getattr(backend, "_initialized", False):
        raise RuntimeError("Backend not initialized")
    s = backend.export_state(env_idx, env_idx + 1)
    m = np.asarray(s["mem"]).reshape(-1)
    cs = np.asarray(s["cart_state"]).reshape(-1)
    from .cartridge import CS

    one = lambda k: int(np.asarray(s[k]).reshape(-1)[0])  # noqa: E731
    rombank = ((int(cs[CS["rom_bank_hi"]]) & 3) << 5) | (int(cs[CS["rom_bank_lo"]]) & 0x7F)
    ram_len = int(backend._spec.ram_byte_length)
    cart_ram = bytes(np.asarray(s["cart_ram"]).reshape(-1)[:ram_len]) if ram_len > 0 else b""
    div_full = one("div_counter") & 0xFFFF
    ly = one("ppu_ly") & 0xFF
    scan_cycle = one("ppu_scanline_cycle")
    lcd_clock = ly * CYCLES_PER_LINE + scan_cycle
    scx, scy, wx, wy = int(m[0xFF43]), int(m[0xFF42]), int(m[0xFF4B]), int(m[0xFF4A])
    params = bytes([scx, scy, wx, wy, 0]) * SCREEN_H
    return PyBoyState(
        version=VERSION_SAVE, bootrom_enabled=int(cs[CS["bootrom_enabled"]]) & 1,
        a=one("a") & 0xFF, f=one("f") & 0xF0, b=one("b") & 0xFF, c=one("c") & 0xFF, d=one("d") & 0xFF,
        e=one("e") & 0xFF, h=one("h") & 0xFF, l_reg=one("l") & 0xFF, sp=one("sp") & 0xFFFF,
        pc=one("pc") & 0xFFFF, ime=one("ime") & 1, halted=one("halted") & 1, stopped=0,
        ie=int(m[0xFFFF]), interrupt_queued=0, if_reg=int(m[0xFF0F]), cpu_cycles=one("cycle_count"),
        vram=bytes(m[0x8000:0xA000]), oam=bytes(m[0xFE00:0xFEA0]), lcdc=int(m[0xFF40]),
        stat=int(m[0xFF41]), ly=ly, lyc=int(m[0xFF45]), scy=scy, scx=scx, wy=wy, wx=wx,
        bgp=int(m[0xFF47]), obp0=int(m[0xFF48]), obp1=int(m[0xFF49]), lcd_clock=lcd_clock,
        lcd_clock_target=lcd_clock + CYCLES_PER_LINE, next_stat_mode=_mode_of(ly, scan_cycle),
        scanline_params=params, wram=bytes(m[0xC000:0xE000]), hram=bytes(m[0xFF80:0xFFFF]),
        io_ports=bytes(m[0xFF00:0xFF4C]), non_io_ram0=bytes(m[0xFEA0:0xFF00]),
        non_io_ram1=bytes(m[0xFF4C:0xFF80]), div=(div_full >> 8) & 0xFF, tima=int(m[0xFF05]),
        tma=int(m[0xFF06]), tac=int(m[0xFF07]), div_counter=div_full & 0xFF, tima_counter=0,
        rombank=rombank, rambank=int(cs[CS["ram_bank"]]) & 0xFF,
        rambank_enabled=int(cs[CS["ram_enable"]]) & 1, memorymodel=int(cs[CS["bank_mode"]]) & 1,
        cart_ram=cart_ram, joypad_directional=0x0F, joypad_standard=0x0F,
        serial_sb=int(m[0xFF01]), serial_sc=int(m[0xFF02]))


def apply_state_to_backend(state: PyBoyState, backend: Any, env_idx: int = 0) -> None:
    """Load ``state`` into env ``env_idx`` (state_io.py:839-1154).

    As in the reference: the env's address-space regions, LCD/timer/interrupt
    registers, CPU registers and cartridge bank registers come from the
    state; the timer-edge, reload and STAT-edge trackers are recomputed;
    cycle_in_frame restarts at 0; the env-0 scanline latches (shared by the
    batch) are seeded from the state's scanline parameters.
    """
    if not getattr(backend, "_initialized", False):
        raise RuntimeError("Backend not initialized")
    from .cartridge import CS

    lo, hi = env_idx, env_idx + 1
    s = backend.export_state(lo, hi)
    m = np.asarray(s["mem"]).reshape(-1).copy()
    cs = np.asarray(s["cart_state"]).reshape(-1).copy()
    cs[CS["bootrom_enabled"]] = 1 if state.bootrom_enabled else 0
    cs[CS["rom_bank_lo"]] = state.rombank & 0xFF
    cs[CS["rom_bank_hi"]] = (state.rombank >> 8) & 0xFF
    cs[CS["ram_bank"]] = state.rambank & 0xFF
    cs[CS["ram_enable"]] = state.rambank_enabled & 1
    cs[CS["bank_mode"]] = state.memorymodel & 1
    cart_ram = np.asarray(s["cart_ram"]).reshape(-1).copy()
    ram_len = int(backend._spec.ram_byte_length)
    if ram_len > 0 and state.cart_ram:
        src = np.frombuffer(state.cart_ram, dtype=np.uint8)[:ram_len]
        cart_ram[:ram_len] = 0
        cart_ram[:src.size] = src

    def put(addr: int, data: bytes) -> None:
        m[addr:addr + len(data)] = np.frombuffer(data, dtype=np.uint8)

    put(0x8000, state.vram)
    put(0xFE00, state.oam)
    put(0xC000, state.wram)
    put(0xFF80, state.hram)
    put(0xFF00, state.io_ports)
    put(0xFEA0, state.non_io_ram0)
    put(0xFF4C, state.non_io_ram1)
    regs = {0xFF0F: state.if_reg, 0xFFFF: state.ie, 0xFF01: state.serial_sb, 0xFF02: state.serial_sc,
            0xFF00: 0xCF, 0xFF04: state.div, 0xFF05: state.tima, 0xFF06: state.tma, 0xFF07: state.tac,
            0xFF40: state.lcdc, 0xFF41: state.stat, 0xFF42: state.scy, 0xFF43: state.scx,
            0xFF44: state.ly, 0xFF45: state.lyc, 0xFF47: state.bgp, 0xFF48: state.obp0,
            0xFF49: state.obp1, 0xFF4A: state.wy, 0xFF4B: state.wx}
    for addr, v in regs.items():
        m[addr] = int(v) & 0xFF

    div_full = ((int(state.div) & 0xFF) << 8) | (int(state.div_counter) & 0xFF)
    tac = int(state.tac)
    prev_in = (div_full >> (9, 3, 5, 7)[tac & 3]) & 1 if tac & 4 else 0
    cycle_count = int(state.cpu_cycles) if state.cpu_cycles != 0 else int(state.lcd_clock)
    cycle_count = max(np.iinfo(np.int64).min, min(np.iinfo(np.int64).max, cycle_count))
    mode = int(state.stat) & 3
    stat_prev = (mode == 0) | ((mode == 1) << 1) | ((mode == 2) << 2) | ((int(state.ly) == int(state.lyc)) << 3)
    scalars = {"a": state.a, "f": state.f, "b": state.b, "c": state.c, "d": state.d, "e": state.e,
               "h": state.h, "l": state.l_reg, "sp": state.sp, "pc": state.pc, "ime": state.ime,
               "ime_delay": 0, "halted": state.halted, "div_counter": div_full, "timer_prev_in": prev_in,
               "tima_reload_pending": 0, "tima_reload_delay": 0, "joyp_select": 0x30,
               "ppu_ly": state.ly, "ppu_scanline_cycle": int(state.lcd_clock) % CYCLES_PER_LINE,
               "cycle_count": cycle_count, "cycle_in_frame": 0,
               "ppu_window_line": state.ly - state.wy if state.ly >= state.wy else 0,
               "ppu_stat_prev": stat_prev}
    new = dict(s)  # every exported field, so the scalar block imports whole
    new.update({"mem": m, "cart_state": cs, "cart_ram": cart_ram})
    for k, v in scalars.items():
        arr = np.asarray(s[k]).reshape(-1).copy()
        arr[0] = v
        new[k] = arr
    latches = None
    if len(state.scanline_params) >= SCREEN_H * 5:
        p = np.frombuffer(state.scanline_params, dtype=np.uint8)[:SCREEN_H * 5].reshape(SCREEN_H, 5)
        y = np.arange(SCREEN_H)
        wy_l = p[:, 3].astype(np.int64)
        latches = {"bg_lcdc": np.full(SCREEN_H, state.lcdc), "bg_scx": p[:, 0], "bg_scy": p[:, 1],
                   "bg_bgp": np.full(SCREEN_H, state.bgp), "win_wx": p[:, 2], "win_wy": p[:, 3],
                   "win_line": np.where(y >= wy_l, (y - wy_l) & 0xFF, 0),
                   "obj_obp0": np.full(SCREEN_H, state.obp0), "obj_obp1": np.full(SCREEN_H, state.obp1)}
        for k, v in latches.items():
            new[f"latch_{k}"] = np.asarray(v, dtype=np.uint8)
    backend.import_state(new, lo, hi)
