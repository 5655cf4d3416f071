"""Every-opcode probe batch: one SM83 instruction per env, then a trap.

TEST INFRASTRUCTURE. Env k starts at the entry of its own 16-byte slot of a
32 KiB ROM-only image with preset registers; the slot holds one instruction
(every unprefixed opcode, every CB-prefixed opcode, and each conditional jump,
call and return once with its condition true and once false). Every other
ROM byte is 0xD3, an unimplemented opcode: the instruction after the probed
one traps (trap kind 1, zero cycles, the env stops), so after one step

* ``trap_pc`` is where the probed instruction sent the PC (its length, or its
  jump target),
* ``cycle_count`` is its cycle count,
* ``instr_count`` is 1,

which ``expected()`` derives from the reference's ISA table
(``src/gbxcule/core/isa_sm83.py``, exported to ``golden/isa_sm83.json``).
STOP and the unimplemented opcodes trap at the slot itself; HALT halts (no
interrupt is enabled) and sleeps out the frame. Jump targets (JP, JR, CALL,
JP (HL), the return address on the stack, the RST vectors) all land on trap
bytes at known places.

``make_fixtures.py`` runs this batch through the reference's own kernel source
for a golden digest; the oracle (CPU) and libgbx (GPU) tests replay it.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

from gbxcule_b200 import cartridge as cart
from gbxcule_b200 import roms
from gbxcule_b200.state import LATCHES, MEM_SIZE, OBS_DIM, SCALARS, SERIAL_MAX

GOLDEN = Path(__file__).resolve().parent / "golden"
TRAP = 0xD3
SLOT0, SLOT = 0x200, 16
TARGET = 8            # jump targets: slot + 8
SP0 = 0xD000          # stack pointer; the return address sits at SP0..SP0+1
REGS = dict(a=0x5A, b=0xC3, c=0x90, d=0xC4, e=0x10, h=0xC2, l=0x00)   # BC, DE, HL in WRAM; (C) = FF90
CONDITIONAL = {0x20, 0x28, 0x30, 0x38, 0xC0, 0xC8, 0xD0, 0xD8, 0xC2, 0xCA, 0xD2, 0xDA, 0xC4, 0xCC, 0xD4, 0xDC}
# flag byte making condition (op >> 3) & 3 (NZ, Z, NC, C) true / false
COND_F = {0: (0x00, 0x80), 1: (0x80, 0x00), 2: (0x00, 0x10), 3: (0x10, 0x00)}


def isa_table() -> dict:
    """The reference's opcode table (exported by golden/make_isa_fixture.py)."""
    return json.loads((GOLDEN / "isa_sm83.json").read_text())


def probes() -> list[dict]:
    """One dict per env: prefix (0/1), opcode, taken (conditionals only)."""
    out = []
    for op in range(256):
        if op == 0xCB:
            continue  # the CB prefix is probed through every CB opcode below
        if op in CONDITIONAL:
            out.append(dict(prefix=0, op=op, taken=True))
            out.append(dict(prefix=0, op=op, taken=False))
        else:
            out.append(dict(prefix=0, op=op, taken=None))
    out.extend(dict(prefix=1, op=op, taken=None) for op in range(256))
    return out


def _operands(op: int, slot: int) -> list[int]:
    """Operand bytes of an unprefixed opcode placed at ``slot``."""
    tgt = slot + TARGET
    if op in (0x18, 0x20, 0x28, 0x30, 0x38):                 # JR: slot + 2 + e = target
        return [TARGET - 2]
    if op in (0xC3, 0xC2, 0xCA, 0xD2, 0xDA, 0xCD, 0xC4, 0xCC, 0xD4, 0xDC):
        return [tgt & 0xFF, tgt >> 8]
    if op == 0x08:                                           # LD (a16),SP
        return [0x00, 0xC5]
    if op in (0xEA, 0xFA):                                   # LD (a16),A / LD A,(a16)
        return [0x00, 0xC6]
    if op in (0xE0, 0xF0):                                   # LDH: HRAM
        return [0x91]
    if op in (0xE8, 0xF8):                                   # SP + e8
        return [0x05]
    if op in (0x01, 0x11, 0x21, 0x31):                       # LD rr,d16
        return [0x34, 0x12]
    return [0x3C]                                            # any d8 (unused bytes are overwritten)


def rom_image() -> bytes:
    """32 KiB ROM-only image: trap bytes everywhere, one probed instruction per slot."""
    rom = bytearray([TRAP]) * 0x8000
    for k, p in enumerate(probes()):
        slot = SLOT0 + SLOT * k
        if p["prefix"]:
            rom[slot:slot + 2] = bytes([0xCB, p["op"]])
        else:
            spec = isa_table()["unprefixed"][p["op"]]
            body = [p["op"]] + _operands(p["op"], slot)
            rom[slot:slot + max(spec["length"], 1)] = bytes(body[:max(spec["length"], 1)])
    rom[0x104:0x150] = bytes(0x4C)
    roms.finalize_header(rom, title="GBXISAPROBE", cart_type=0x00, rom_code=0x00, ram_code=0x00)
    return bytes(rom)


def initial_state(rom: bytes) -> dict:
    """Per-env state (``export_state`` layout) that puts env k at its slot."""
    ps = probes()
    n = len(ps)
    spec = cart.parse_cartridge_header(rom)
    s = {name: np.zeros(n, dtype=dt) for name, dt in SCALARS}
    mem = np.zeros((n, MEM_SIZE), dtype=np.uint8)
    cs = np.zeros((n, cart.CART_STATE_STRIDE), dtype=np.int32)
    cs[:, cart.CS["mbc_kind"]] = spec.mbc_kind
    cs[:, cart.CS["rom_bank_lo"]] = 1          # boot ROM off (bootrom_enabled = 0)
    s["joyp_select"][:] = 0x30
    for k, p in enumerate(ps):
        slot = SLOT0 + SLOT * k
        s["pc"][k] = slot
        s["sp"][k] = SP0
        for r, v in REGS.items():
            s[r][k] = v
        if not p["prefix"] and p["op"] == 0xE9:               # JP (HL)
            s["h"][k], s["l"][k] = (slot + TARGET) >> 8, (slot + TARGET) & 0xFF
        s["f"][k] = 0x00
        if p["taken"] is not None:
            s["f"][k] = COND_F[(p["op"] >> 3) & 3][0 if p["taken"] else 1]
        ret = slot + TARGET
        mem[k, SP0], mem[k, SP0 + 1] = ret & 0xFF, ret >> 8
    s["mem"] = mem.reshape(-1)
    s["cart_state"] = cs.reshape(-1)
    s["cart_ram"] = np.zeros(n * max(spec.ram_byte_length, 1), dtype=np.uint8)
    s["serial_buf"] = np.zeros(n * SERIAL_MAX, dtype=np.uint8)
    s["obs"] = np.zeros(n * OBS_DIM, dtype=np.float32)
    s["reward"] = np.zeros(n, dtype=np.float32)
    for k in LATCHES:
        s[f"latch_{k}"] = np.zeros(144, dtype=np.uint8)
    return s


def expected() -> list[dict]:
    """Per env, from the ISA table: trap_pc, cycle_count, instr_count (None for HALT)."""
    t = isa_table()
    out = []
    for k, p in enumerate(probes()):
        slot = SLOT0 + SLOT * k
        op = p["op"]
        if p["prefix"]:
            spec = t["cb"][op]
            out.append(dict(trap_pc=slot + 2, cycles=spec["cycles"][0], instr=1))
            continue
        spec = t["unprefixed"][op]
        if not spec["implemented"]:                           # STOP, illegal: trap here
            out.append(dict(trap_pc=slot, cycles=0, instr=0))
        elif op == 0x76:                                      # HALT
            out.append(dict(trap_pc=None, cycles=None, instr=None, pc=slot + 1, halted=1))
        elif op in (0xC7, 0xCF, 0xD7, 0xDF, 0xE7, 0xEF, 0xF7, 0xFF):   # RST: vector holds a trap
            out.append(dict(trap_pc=op & 0x38, cycles=spec["cycles"][0], instr=1))
        elif op in (0x18, 0xC3, 0xCD, 0xC9, 0xD9, 0xE9):     # unconditional jumps
            out.append(dict(trap_pc=slot + TARGET, cycles=spec["cycles"][0], instr=1))
        elif p["taken"] is not None:
            cyc = spec["cycles"][0] if p["taken"] else spec["cycles"][1]
            out.append(dict(trap_pc=slot + TARGET if p["taken"] else slot + spec["length"], cycles=cyc, instr=1))
        else:
            out.append(dict(trap_pc=slot + spec["length"], cycles=spec["cycles"][0], instr=1))
    return out


def check(state: dict) -> list[str]:
    """Mismatches between a stepped probe batch and the ISA table."""
    bad = []
    for k, (p, e) in enumerate(zip(probes(), expected())):
        name = f"{'CB ' if p['prefix'] else ''}{p['op']:02X}" + ("" if p["taken"] is None else
                                                                f" ({'taken' if p['taken'] else 'not taken'})")
        if e["trap_pc"] is None:
            if int(state["pc"][k]) != e["pc"] or int(state["halted"][k]) != 1:
                bad.append(f"{name}: pc {int(state['pc'][k]):#06x} halted {int(state['halted'][k])}")
            continue
        got = (int(state["trap_pc"][k]), int(state["cycle_count"][k]), int(state["instr_count"][k]),
               int(state["trap_flag"][k]))
        want = (e["trap_pc"], e["cycles"], e["instr"], 1)
        if got != want:
            bad.append(f"{name}: (trap_pc, cycles, instr, trap) {got} != {want}")
    return bad
