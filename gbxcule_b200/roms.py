"""Synthetic, seeded Game Boy ROMs and the from-source boot stub.

Everything here is generated from a seed by code in this file; no ROM or boot
ROM image from elsewhere is read. The generators implement the five workload
contracts of the benchmark (config 1..5):

* ``config1_rom``  32 KiB, no MBC, LCD off: a loop of 2,000 uniformly drawn
  implemented SM83 opcodes (CB-prefixed included) whose memory operands are
  forced into WRAM, with a joypad read + branch every 64 ops.
* ``config2_rom``  the same loop with the PPU on (LCDC=0xE3), random VRAM tiles,
  random BG/window maps, 40 random sprites, SCX/SCY bumped by a VBlank handler.
* ``config3_rom``  interrupt/timer heavy: TAC cycled through the four clocks,
  timer + STAT(LYC) + VBlank IRQs, HALT under IME=0 and IME=1, EI/DI, OAM DMA
  from a random WRAM page once per frame.
* ``config4_rom``  MBC3 + 32 KiB RAM, 64 x 16 KiB banks of seeded code that
  bank-switch every ~256 instructions, touch cart RAM, and dispatch through a
  16-entry joypad jump table.
* ``config5_rom``  the config-4 cartridge with the config-2 PPU settings.

The boot stub is a 256-byte SM83 program that sets DMG post-boot registers and
writes FF50 from its last two bytes, so execution falls through to 0x0100.
The reference emulator (bkase/gbxcule) maps its boot ROM over 0x0000-0x00FF
until FF50 is written (``src/gbxcule/kernels/cpu_step_builder.py:561-564``,
``:724-727``); this stub plays that role for every implementation here.
"""

from __future__ import annotations

import numpy as np

ROM_BANK = 0x4000

# Register encodings used by the SM83 opcode matrix (B C D E H L (HL) A).
R8 = {"b": 0, "c": 1, "d": 2, "e": 3, "h": 4, "l": 5, "hl": 6, "a": 7}
# 16-bit pairs as encoded in PUSH/POP (AF last) and LD rr,d16 (SP last).
PUSHPOP = {"bc": 0, "de": 1, "hl": 2, "af": 3}
RR = {"bc": 0, "de": 1, "hl": 2, "sp": 3}
COND = {"nz": 0, "z": 1, "nc": 2, "c": 3}

# Opcodes the reference marks unimplemented (they trap), plus the CB prefix.
ILLEGAL = frozenset({0xD3, 0xDB, 0xDD, 0xE3, 0xE4, 0xEB, 0xEC, 0xED, 0xF4, 0xFC, 0xFD})
STOP = 0x10
HALT = 0x76
PREFIX_CB = 0xCB

# SP for the synthetic programs; data stores stay below 0xDF00.
SP_BASE = 0xDFF0


def boot_stub() -> bytes:
    """Return the 256-byte boot stub (from source, see module docstring)."""
    code = bytearray(0x100)
    prog = [
        0x31, 0xFE, 0xFF,  # LD SP,0xFFFE
        0x21, 0xB0, 0x01,  # LD HL,0x01B0
        0xE5,              # PUSH HL
        0xF1,              # POP AF        -> A=0x01 F=0xB0
        0x01, 0x13, 0x00,  # LD BC,0x0013
        0x11, 0xD8, 0x00,  # LD DE,0x00D8
        0x21, 0x4D, 0x01,  # LD HL,0x014D
        0xC3, 0xFE, 0x00,  # JP 0x00FE
    ]
    code[: len(prog)] = bytes(prog)
    code[0xFE] = 0xE0  # LDH (0x50),A  -> boot ROM off, PC falls to 0x0100
    code[0xFF] = 0x50
    return bytes(code)


class Asm:
    """Tiny two-pass SM83 assembler: raw bytes plus label fixups."""

    def __init__(self, size: int) -> None:
        self.buf = bytearray(size)
        self.pos = 0
        self.labels: dict[str, int] = {}
        self._abs16: list[tuple[int, str]] = []
        self._rel8: list[tuple[int, str]] = []

    # -- layout -----------------------------------------------------------
    def org(self, addr: int) -> None:
        self.pos = addr

    def label(self, name: str) -> None:
        if name in self.labels:
            raise ValueError(f"duplicate label {name}")
        self.labels[name] = self.pos

    def db(self, *vals: int) -> None:
        for v in vals:
            if self.pos >= len(self.buf):
                raise ValueError("ROM overflow")
            self.buf[self.pos] = v & 0xFF
            self.pos += 1

    def dw_label(self, name: str) -> None:
        self._abs16.append((self.pos, name))
        self.db(0, 0)

    # -- instructions with label operands -----------------------------------
    def op_abs(self, opcode: int, name: str) -> None:
        self.db(opcode)
        self.dw_label(name)

    def jp(self, name: str, cond: str | None = None) -> None:
        self.op_abs(0xC3 if cond is None else 0xC2 | (COND[cond] << 3), name)

    def call(self, name: str, cond: str | None = None) -> None:
        self.op_abs(0xCD if cond is None else 0xC4 | (COND[cond] << 3), name)

    def jr(self, name: str, cond: str | None = None) -> None:
        self.db(0x18 if cond is None else 0x20 | (COND[cond] << 3))
        self._rel8.append((self.pos, name))
        self.db(0)

    def ld_rr(self, rr: str, value: int | str) -> None:
        if isinstance(value, str):
            self.op_abs(0x01 | (RR[rr] << 4), value)
        else:
            self.db(0x01 | (RR[rr] << 4), value & 0xFF, (value >> 8) & 0xFF)

    # -- plain instructions --------------------------------------------------
    def ld_r_d8(self, r: str, v: int) -> None:
        self.db(0x06 | (R8[r] << 3), v)

    def ldh_store(self, a8: int) -> None:  # LDH (a8),A
        self.db(0xE0, a8)

    def ldh_load(self, a8: int) -> None:  # LDH A,(a8)
        self.db(0xF0, a8)

    def ld_a16_a(self, addr: int) -> None:
        self.db(0xEA, addr & 0xFF, addr >> 8)

    def ld_a_a16(self, addr: int) -> None:
        self.db(0xFA, addr & 0xFF, addr >> 8)

    def push(self, rr: str) -> None:
        self.db(0xC5 | (PUSHPOP[rr] << 4))

    def pop(self, rr: str) -> None:
        self.db(0xC1 | (PUSHPOP[rr] << 4))

    def finish(self) -> bytes:
        for at, name in self._abs16:
            tgt = self.labels[name]
            self.buf[at] = tgt & 0xFF
            self.buf[at + 1] = (tgt >> 8) & 0xFF
        for at, name in self._rel8:
            off = self.labels[name] - (at + 1)
            if not -128 <= off <= 127:
                raise ValueError(f"JR to {name} out of range ({off})")
            self.buf[at] = off & 0xFF
        return bytes(self.buf)


def finalize_header(rom: bytearray, *, title: str, cart_type: int,
                    rom_code: int, ram_code: int) -> bytes:
    """Write entry point, title, cart fields and both checksums."""
    rom[0x100:0x104] = bytes([0x00, 0xC3, 0x50, 0x01])  # NOP; JP 0x0150
    t = title.encode("ascii")[:15]
    rom[0x134:0x134 + len(t)] = t
    rom[0x147] = cart_type
    rom[0x148] = rom_code
    rom[0x149] = ram_code
    x = 0
    for b in rom[0x134:0x14D]:
        x = (x - b - 1) & 0xFF
    rom[0x14D] = x
    rom[0x14E] = 0
    rom[0x14F] = 0
    g = sum(rom) & 0xFFFF
    rom[0x14E] = g >> 8
    rom[0x14F] = g & 0xFF
    return bytes(rom)


# ---------------------------------------------------------------------------
# Opcode pool for the random loop
# ---------------------------------------------------------------------------

def _loop_pool(*, allow_di: bool) -> list[tuple[int, int]]:
    """(prefix, opcode) pairs drawn uniformly by the loop generator.

    prefix 0 = unprefixed, 1 = CB-prefixed.  STOP, HALT, the CB prefix byte and
    the unimplemented opcodes are excluded (they trap, or never wake without an
    interrupt source).
    """
    pool = []
    for op in range(256):
        if op in ILLEGAL or op in (STOP, HALT, PREFIX_CB):
            continue
        if op == 0xF3 and not allow_di:
            continue
        pool.append((0, op))
    pool.extend((1, op) for op in range(256))
    return pool


def _r8_name(code: int) -> str:
    return "bchl?a"[code] if code != 6 else "hl"


class _LoopGen:
    """Emits guarded units for randomly drawn opcodes into an ``Asm``.

    Every unit leaves SP at ``SP_BASE`` and keeps all data accesses inside
    WRAM C000-DEFF (or HRAM for the LDH forms), so any unit boundary is a safe
    branch target.
    """

    def __init__(self, asm: Asm, rng: np.random.Generator, prefix: str,
                 ram_window: tuple[int, int] = (0xC0, 0xDE)) -> None:
        self.a = asm
        self.rng = rng
        self.prefix = prefix
        self.n_units = 0
        self.ram_lo, self.ram_hi = ram_window

    def _r(self, lo: int, hi: int) -> int:
        return int(self.rng.integers(lo, hi + 1))

    def unit_label(self, k: int) -> str:
        return f"{self.prefix}_u{k}"

    def _hi_guard(self, reg: str, lo_pad: int = 0, hi_pad: int = 0) -> None:
        self.a.ld_r_d8(reg, self._r(self.ram_lo + lo_pad, self.ram_hi - hi_pad))

    def emit(self, pref: int, op: int) -> None:
        a = self.a
        k = self.n_units
        a.label(self.unit_label(k))
        nxt = self.unit_label(k + 1)
        self.n_units += 1
        if pref == 1:
            if (op & 7) == 6:
                self._hi_guard("h")
            a.db(0xCB, op)
            return
        hi, lo = op >> 4, op & 0xF
        # (HL) operands -----------------------------------------------------
        uses_hl = (
            op in (0x34, 0x35, 0x36)
            or (0x40 <= op <= 0x7F and ((op & 7) == 6 or (op >> 3) & 7 == 6))
            or (0x80 <= op <= 0xBF and (op & 7) == 6)
        )
        if uses_hl:
            self._hi_guard("h")
            a.db(op)
            if op == 0x36:
                a.db(self._r(0, 255))
            return
        if op in (0x22, 0x2A, 0x32, 0x3A):  # LDI/LDD
            self._hi_guard("h", 1, 1)
            a.db(op)
            return
        if op in (0x02, 0x0A):
            self._hi_guard("b")
            a.db(op)
            return
        if op in (0x12, 0x1A):
            self._hi_guard("d")
            a.db(op)
            return
        if op in (0xEA, 0xFA):
            addr = self._r(self.ram_lo << 8, (self.ram_hi << 8) | 0xFF)
            a.db(op, addr & 0xFF, addr >> 8)
            return
        if op == 0x08:  # LD (a16),SP
            addr = self._r(self.ram_lo << 8, (self.ram_hi << 8) | 0xFE)
            a.db(op, addr & 0xFF, addr >> 8)
            return
        if op in (0xE0, 0xF0):  # LDH (a8) forms stay in HRAM
            a.db(op, self._r(0x80, 0xFD))
            return
        if op in (0xE2, 0xF2):
            a.ld_r_d8("c", self._r(0x80, 0xFD))
            a.db(op)
            return
        # stack ---------------------------------------------------------------
        if op == 0x31:
            a.db(op, SP_BASE & 0xFF, SP_BASE >> 8)
            return
        if op == 0xF9:
            a.ld_rr("hl", SP_BASE)
            a.db(op)
            return
        if op == 0x33:
            a.db(0x33, 0x3B)
            return
        if op == 0x3B:
            a.db(0x3B, 0x33)
            return
        if op == 0xE8:
            e = self._r(-127, 127)
            a.db(0xE8, e & 0xFF, 0xE8, (-e) & 0xFF)
            return
        if op in (0xC5, 0xD5, 0xE5, 0xF5):
            a.db(op)
            a.pop(["bc", "de", "hl", "af"][self._r(0, 3)])
            return
        if op in (0xC1, 0xD1, 0xE1, 0xF1):
            a.push(["bc", "de", "hl", "af"][self._r(0, 3)])
            a.db(op)
            return
        # control flow -------------------------------------------------------
        if op == 0x18:
            pad = self._r(0, 3)
            a.db(0x18, pad)
            a.db(*[self._r(0, 255) for _ in range(pad)])  # never executed
            return
        if op in (0x20, 0x28, 0x30, 0x38):
            pad = self._r(0, 3)
            a.db(op, pad)
            a.db(*([0x00] * pad))
            return
        if op == 0xC3 or op in (0xC2, 0xCA, 0xD2, 0xDA):
            a.op_abs(op, nxt)
            return
        if op == 0xE9:
            a.ld_rr("hl", nxt)
            a.db(0xE9)
            return
        if op == 0xCD or op in (0xC4, 0xCC, 0xD4, 0xDC):
            a.op_abs(op, "ret_stub")
            return
        if op in (0xC9, 0xD9, 0xC0, 0xC8, 0xD0, 0xD8):
            body = f"{self.prefix}_r{k}"
            a.call(body)
            a.jr(nxt)
            a.label(body)
            a.db(op)
            if op not in (0xC9, 0xD9):
                a.db(0xC9)
            return
        if (op & 0xC7) == 0xC7:  # RST n -> RET at the vector
            a.db(op)
            return
        # plain register ops, with random immediates ---------------------------
        a.db(op)
        if op in (0x06, 0x0E, 0x16, 0x1E, 0x26, 0x2E, 0x3E) or (hi >= 0xC and lo in (0x6, 0xE)):
            a.db(self._r(0, 255))
        elif op == 0xF8:
            a.db(self._r(0, 255))
        elif op in (0x01, 0x11, 0x21):
            v = self._r(0, 0xFFFF)
            a.db(v & 0xFF, v >> 8)

    def joypad_check(self, k: int, skip_max: int = 8) -> None:
        """Write JOYP select, read it back, branch on one input bit."""
        a = self.a
        sel = 0x20 if self._r(0, 1) == 0 else 0x10
        bit = self._r(0, 3)
        a.ld_r_d8("a", sel)
        a.ldh_store(0x00)
        a.ldh_load(0x00)
        a.db(0xE6, 1 << bit)  # AND mask
        tgt = self.unit_label(k + self._r(1, skip_max))
        a.jp(tgt, "z")


def _common_vectors(a: Asm) -> None:
    """RET at every RST vector and a shared RET stub for CALL units."""
    for v in range(0, 0x40, 8):
        a.org(v)
        a.db(0xC9)
    a.org(0x68)
    a.label("ret_stub")
    a.db(0xC9)


def _emit_loop(a: Asm, rng: np.random.Generator, *, n_ops: int, prefix: str,
               allow_di: bool, joy_every: int = 64,
               ram_window: tuple[int, int] = (0xC0, 0xDE)) -> _LoopGen:
    gen = _LoopGen(a, rng, prefix, ram_window)
    pool = _loop_pool(allow_di=allow_di)
    picks = rng.integers(0, len(pool), size=n_ops)
    for i in range(n_ops):
        if i > 0 and i % joy_every == 0:
            gen.joypad_check(gen.n_units)
        gen.emit(*pool[int(picks[i])])
    # pad labels the last joypad checks may target
    for _ in range(16):
        a.label(gen.unit_label(gen.n_units))
        gen.n_units += 1
    return gen


def _random_regs(a: Asm, rng: np.random.Generator) -> None:
    for rr in ("bc", "de", "hl"):
        a.ld_rr(rr, int(rng.integers(0, 0x10000)))
    a.ld_r_d8("a", int(rng.integers(0, 256)))


def config1_rom(seed: int = 1, n_ops: int = 2000) -> bytes:
    """Config 1: LCD-off random-opcode loop (32 KiB, ROM only)."""
    rng = np.random.default_rng(seed)
    a = Asm(0x8000)
    _common_vectors(a)
    a.org(0x150)
    a.ld_rr("sp", SP_BASE)
    _random_regs(a, rng)
    a.label("loop")
    _emit_loop(a, rng, n_ops=n_ops, prefix="L", allow_di=True)
    a.jp("loop")
    rom = bytearray(a.finish())
    return finalize_header(rom, title="GBXB200 C1", cart_type=0x00, rom_code=0x00, ram_code=0x00)


def _copy_block(a: Asm, src_label: str, dst: int, count: int, tag: str) -> None:
    """Byte copy ROM[src_label..] -> dst using HL/DE/BC (count <= 0xFFFF)."""
    a.ld_rr("hl", src_label)
    a.ld_rr("de", dst)
    a.ld_rr("bc", count)
    a.label(f"cp_{tag}")
    a.db(0x2A)        # LD A,(HL+)
    a.db(0x12)        # LD (DE),A
    a.db(0x13)        # INC DE
    a.db(0x0B)        # DEC BC
    a.db(0x78)        # LD A,B
    a.db(0xB1)        # OR C
    a.jr(f"cp_{tag}", "nz")


def _ppu_setup(a: Asm, rng: np.random.Generator, data_at: int) -> int:
    """Emit code that loads random VRAM/OAM/palettes and turns the LCD on.

    Random data blocks are laid out from ``data_at``; returns the end address.
    """
    vram = rng.integers(0, 256, size=0x1800, dtype=np.uint8)   # tile data 8000-97FF
    maps = rng.integers(0, 256, size=0x800, dtype=np.uint8)    # maps 9800-9FFF
    oam = np.zeros(160, dtype=np.uint8)
    for s in range(40):
        oam[4 * s + 0] = rng.integers(16, 160)   # y in [16, 159]
        oam[4 * s + 1] = rng.integers(8, 168)    # x in [8, 167]
        oam[4 * s + 2] = rng.integers(0, 256)
        oam[4 * s + 3] = rng.integers(0, 256)
    _copy_block(a, "vram_data", 0x8000, 0x1800, "vram")
    _copy_block(a, "map_data", 0x9800, 0x800, "maps")
    _copy_block(a, "oam_data", 0xFE00, 160, "oam")
    for reg in (0x47, 0x48, 0x49):               # BGP OBP0 OBP1
        a.ld_r_d8("a", int(rng.integers(0, 256)))
        a.ldh_store(reg)
    a.ld_r_d8("a", int(rng.integers(0, 144)))     # WY
    a.ldh_store(0x4A)
    a.ld_r_d8("a", int(rng.integers(7, 167)))     # WX
    a.ldh_store(0x4B)
    here = a.pos
    a.org(data_at)
    a.label("vram_data")
    a.db(*vram.tolist())
    a.label("map_data")
    a.db(*maps.tolist())
    a.label("oam_data")
    a.db(*oam.tolist())
    end = a.pos
    a.org(here)
    return end


def config2_rom(seed: int = 2, n_ops: int = 2000) -> bytes:
    """Config 2: config-1 loop with the PPU on (LCDC=0xE3), VBlank scrolls."""
    rng = np.random.default_rng(seed)
    a = Asm(0x8000)
    _common_vectors(a)
    # VBlank handler: SCX++, SCY++ (preserves AF), RETI.
    a.org(0x40)
    a.db(0xF5, 0xF0, 0x43, 0x3C, 0xE0, 0x43, 0xF0, 0x42, 0x3C, 0xE0, 0x42, 0xF1, 0xD9)
    a.org(0x150)
    a.ld_rr("sp", SP_BASE)
    _ppu_setup(a, rng, data_at=0x5000)
    a.ld_r_d8("a", 0x01)   # IE = VBlank
    a.ldh_store(0xFF)
    a.ld_r_d8("a", 0xE3)   # LCD on
    a.ldh_store(0x40)
    a.db(0xFB)             # EI
    _random_regs(a, rng)
    a.label("loop")
    _emit_loop(a, rng, n_ops=n_ops, prefix="L", allow_di=False)
    a.jp("loop")
    if a.pos > 0x5000:
        raise ValueError("config2 code overlaps its data block")
    rom = bytearray(a.finish())
    return finalize_header(rom, title="GBXB200 C2", cart_type=0x00, rom_code=0x00, ram_code=0x00)


def config3_rom(seed: int = 3, n_ops: int = 1500) -> bytes:
    """Config 3: timer/STAT/VBlank IRQs, HALT (IME 0/1), EI/DI, per-frame DMA."""
    rng = np.random.default_rng(seed)
    a = Asm(0x8000)
    _common_vectors(a)
    # VBlank: OAM DMA from a WRAM page picked by a frame counter at C000.
    a.org(0x40)
    a.jp("isr_vblank")
    a.org(0x48)
    a.jp("isr_stat")
    a.org(0x50)
    a.jp("isr_timer")
    a.org(0x150)
    a.ld_rr("sp", SP_BASE)
    a.ld_r_d8("a", int(rng.integers(0, 256)))  # TMA
    a.ldh_store(0x06)
    a.ld_r_d8("a", 0x04)                       # TAC = enabled, 4096 Hz
    a.ldh_store(0x07)
    a.ld_r_d8("a", int(rng.integers(0, 154)))  # LYC
    a.ldh_store(0x45)
    a.ld_r_d8("a", 0x40)                       # STAT: LYC interrupt enable
    a.ldh_store(0x41)
    a.ld_r_d8("a", 0x07)                       # IE: VBlank | STAT | Timer
    a.ldh_store(0xFF)
    a.ld_r_d8("a", 0x91)                       # LCD on
    a.ldh_store(0x40)
    a.db(0xFB)                                 # EI
    _random_regs(a, rng)
    a.label("loop")
    gen = _LoopGen(a, rng, "L")
    pool = _loop_pool(allow_di=True)
    picks = rng.integers(0, len(pool), size=n_ops)
    for i in range(n_ops):
        if i > 0 and i % 64 == 0:
            gen.joypad_check(gen.n_units)
        if i % 50 == 25:
            a.label(gen.unit_label(gen.n_units))
            gen.n_units += 1
            if rng.integers(0, 2) == 0:
                a.db(0xFB, 0x76, 0x00)        # EI; HALT; NOP
            else:
                a.db(0xF3, 0x76, 0x00, 0xFB)  # DI; HALT; NOP (skipped on wake); EI
            continue
        gen.emit(*pool[int(picks[i])])
    for _ in range(16):
        a.label(gen.unit_label(gen.n_units))
        gen.n_units += 1
    a.jp("loop")
    # ISRs (preserve AF/HL)
    pages = rng.integers(0xC0, 0xDF, size=16, dtype=np.uint8)
    a.label("isr_vblank")
    a.db(0xF5, 0xE5)                           # PUSH AF; PUSH HL
    a.ld_rr("hl", 0xDF00)                      # frame counter
    a.db(0x34)                                 # INC (HL)
    a.db(0x7E)                                 # LD A,(HL)
    a.db(0xE6, 0x0F)                           # AND 0x0F
    a.db(0xC6, 0)                              # ADD A,lo(page_table) (patched)
    patch_at = a.pos - 1
    a.db(0x6F)                                 # LD L,A
    a.db(0x26, 0)                              # LD H,hi(page_table) (patched)
    patch_hi = a.pos - 1
    a.db(0x7E)                                 # LD A,(HL)
    a.ldh_store(0x46)                          # DMA
    a.db(0xE1, 0xF1, 0xD9)                     # POP HL; POP AF; RETI
    a.label("isr_stat")
    a.db(0xF5)
    a.ldh_load(0x45)
    a.db(0xC6, int(rng.integers(1, 40)))        # LYC += k
    a.db(0xFE, 154)
    a.jr("stat_ok", "c")
    a.db(0xD6, 154)
    a.label("stat_ok")
    a.ldh_store(0x45)
    a.db(0xF1, 0xD9)
    a.label("isr_timer")
    a.db(0xF5)
    a.ldh_load(0x07)
    a.db(0x3C, 0xE6, 0x03, 0xF6, 0x04)        # INC A; AND 3; OR 4
    a.ldh_store(0x07)
    a.db(0xF1, 0xD9)
    # 16-entry DMA page table, 256-aligned within one page
    a.pos = (a.pos + 0xFF) & ~0xFF
    a.label("page_table")
    a.db(*pages.tolist())
    rom = bytearray(a.finish())
    tbl = a.labels["page_table"]
    rom[patch_at] = tbl & 0xFF
    rom[patch_hi] = tbl >> 8
    return finalize_header(rom, title="GBXB200 C3", cart_type=0x00, rom_code=0x00, ram_code=0x00)


def _mbc3_rom(seed: int, *, ppu: bool, n_banks: int = 64, ops_per_bank: int = 256) -> bytes:
    """Config 4/5 cartridge: MBC3+RAM+BATTERY, 1 MiB ROM, 32 KiB RAM."""
    rng = np.random.default_rng(seed)
    a = Asm(n_banks * ROM_BANK)
    _common_vectors(a)
    if ppu:
        a.org(0x40)
        a.db(0xF5, 0xF0, 0x43, 0x3C, 0xE0, 0x43, 0xF0, 0x42, 0x3C, 0xE0, 0x42, 0xF1, 0xD9)
    a.org(0x150)
    a.ld_rr("sp", SP_BASE)
    a.ld_r_d8("a", 0x0A)       # cart RAM enable
    a.ld_a16_a(0x0000)
    if ppu:
        _ppu_setup(a, rng, data_at=0x1000)
        a.ld_r_d8("a", 0x01)
        a.ldh_store(0xFF)
        a.ld_r_d8("a", 0xE3)
        a.ldh_store(0x40)
        a.db(0xFB)
    _random_regs(a, rng)
    a.ld_r_d8("a", 0x01)
    a.ld_a16_a(0xC100)         # next-bank cursor in WRAM
    # Trampoline: read joypad (both halves) -> 16-way jump table -> pick bank.
    a.label("tramp")
    a.ld_r_d8("a", 0x20)
    a.ldh_store(0x00)
    a.ldh_load(0x00)
    a.db(0xE6, 0x0F)           # AND 0x0F : d-pad nibble
    a.db(0x87)                 # ADD A,A  : *2 (table of words)
    a.db(0x5F)                 # LD E,A
    a.db(0x16, 0x00)           # LD D,0
    a.ld_rr("hl", "jtab")
    a.db(0x19)                 # ADD HL,DE
    a.db(0x2A, 0x66, 0x6F)     # LD A,(HL+); LD H,(HL); LD L,A
    a.db(0xE9)                 # JP (HL)
    a.label("jtab")
    for t in range(16):
        a.dw_label(f"jt{t}")
    for t in range(16):
        a.label(f"jt{t}")
        step = int(rng.integers(1, n_banks))
        a.ld_a_a16(0xC100)
        a.db(0xC6, step)                   # ADD A,step
        a.db(0xE6, n_banks - 1)            # AND banks-1
        a.jr(f"jt{t}_nz", "nz")
        a.db(0x3C)                         # INC A (bank 0 -> 1)
        a.label(f"jt{t}_nz")
        a.ld_a16_a(0xC100)
        a.ld_a16_a(0x2100)                 # ROM bank select
        a.db(0xE6, 0x03)
        a.ld_a16_a(0x4100)                 # RAM bank select (0..3)
        a.jp("bank_entry")
    a.label("bank_entry_pad")
    tramp_end = a.pos
    if ppu and tramp_end > 0x1000:
        raise ValueError("bank-0 code overlaps PPU data")
    for bank in range(1, n_banks):
        a.org(bank * ROM_BANK)
        if bank == 1:
            a.label("bank_entry_phys")
        gen = _LoopGen(a, rng, f"B{bank}", ram_window=(0xA0, 0xDE))
        pool = _loop_pool(allow_di=not ppu)
        picks = rng.integers(0, len(pool), size=ops_per_bank)
        for i in range(ops_per_bank):
            if i > 0 and i % 64 == 0:
                gen.joypad_check(gen.n_units)
            gen.emit(*pool[int(picks[i])])
        for _ in range(16):
            a.label(gen.unit_label(gen.n_units))
            gen.n_units += 1
        a.jp("tramp")
    # labels inside banks are physical offsets; CPU addresses are 0x4000 + off
    rom = bytearray(a.buf)
    lab = a.labels
    lab["bank_entry"] = 0x4000
    for at, name in a._abs16:
        tgt = lab[name]
        if tgt >= 0x8000:
            tgt = 0x4000 + (tgt % ROM_BANK)
        rom[at] = tgt & 0xFF
        rom[at + 1] = tgt >> 8
    for at, name in a._rel8:
        off = lab[name] - (at + 1)
        if not -128 <= off <= 127:
            raise ValueError(f"JR to {name} out of range")
        rom[at] = off & 0xFF
    title = "GBXB200 C5" if ppu else "GBXB200 C4"
    return finalize_header(rom, title=title, cart_type=0x13, rom_code=0x05, ram_code=0x03)


def config4_rom(seed: int = 4) -> bytes:
    """Config 4: MBC3 banked code + cart RAM + joypad jump table."""
    return _mbc3_rom(seed, ppu=False)


def config5_rom(seed: int = 5) -> bytes:
    """Config 5: config-4 cartridge with config-2 PPU settings."""
    return _mbc3_rom(seed, ppu=True)


CONFIG_ROMS = {1: config1_rom, 2: config2_rom, 3: config3_rom, 4: config4_rom, 5: config5_rom}


# ---------------------------------------------------------------------------
# Seeded action traces
# ---------------------------------------------------------------------------

def uniform_actions(rng: np.random.Generator, num_envs: int, n_actions: int = 9) -> np.ndarray:
    """Uniform action indices in [0, n_actions) (configs 1, 2, 4)."""
    return rng.integers(0, n_actions, size=num_envs).astype(np.int32)


def bernoulli_actions(rng: np.random.Generator, num_envs: int, p: float = 0.3) -> np.ndarray:
    """Config 3: 8 Bernoulli(p) buttons per env, projected to one index.

    The reference ABI carries a single action index per env, so the chord is
    projected to the first pressed button in codec order A, B, START, UP,
    DOWN, LEFT, RIGHT (SELECT has no index); no press -> 0 (NOOP).
    """
    presses = rng.random((num_envs, 8)) < p
    # columns: A B SELECT START UP DOWN LEFT RIGHT
    order = [(0, 1), (1, 2), (3, 3), (4, 4), (5, 5), (6, 6), (7, 7)]
    out = np.zeros(num_envs, dtype=np.int32)
    done = np.zeros(num_envs, dtype=bool)
    for col, idx in order:
        hit = presses[:, col] & ~done
        out[hit] = idx
        done |= hit
    return out
