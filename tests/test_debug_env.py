"""Debug-trap settings parsed from the environment as the reference parses
them (src/gbxcule/kernels/cpu_step.py:85-105): ``int(text, 0)``, masks to 16
bits for addresses, negative instruction limits clamp to 0, unparsable text
turns a check off, and any non-empty GBXCULE_TRAP_RST38 turns that check on.
"""

from __future__ import annotations

import pytest

from gbxcule_b200.debug_traps import DebugTraps, read_debug_env


def test_unset_means_every_check_off():
    t = read_debug_env({})
    assert t == DebugTraps() and not t.active


@pytest.mark.parametrize("text, want", [
    ("0x0150", 0x0150), ("336", 336), ("0o17", 15), ("0b101", 5),
    ("0x10150", 0x0150),          # masked to 16 bits
    ("-1", 0xFFFF),               # two's complement, then masked
    ("010", 0),                   # int("010", 0) is a ValueError: off
    ("bogus", 0), ("", 0),
])
def test_addresses(text, want):
    assert read_debug_env({"GBXCULE_TRAP_PC": text}).trap_pc == want
    assert read_debug_env({"GBXCULE_WATCH_ADDR": text}).watch_addr == want


@pytest.mark.parametrize("text, want", [("30000", 30000), ("0x10", 16), ("-5", 0), ("1e3", 0), ("", 0)])
def test_instruction_limit(text, want):
    assert read_debug_env({"GBXCULE_MAX_INSTR": text}).max_instr == want


@pytest.mark.parametrize("text, want", [("1", 1), ("0", 1), ("no", 1), ("", 0)])
def test_rst38_is_on_for_any_nonempty_value(text, want):
    t = read_debug_env({"GBXCULE_TRAP_RST38": text})
    assert t.trap_rst38 == want and t.active == bool(want)
