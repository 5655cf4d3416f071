"""Debug traps, configured from the environment as the reference does.

The reference compiles four optional checks into its step kernel from
environment variables read when the kernel is fetched
(src/gbxcule/kernels/cpu_step.py:85-105): ``GBXCULE_TRAP_PC`` (trap before
executing at that PC, kind 5), ``GBXCULE_TRAP_RST38`` (trap on RST 38 outside
0x0038, kind 3, or on a jump into FE00-FFFF, kind 4), ``GBXCULE_MAX_INSTR``
(trap after that many instructions in one launch, kind 6) and
``GBXCULE_WATCH_ADDR`` (trap when that byte changes, kind 7). Values parse
with Python's ``int(text, 0)``; unparsable values turn a check off; 0 means
off. The reference reads them when a backend fetches its kernel
(warp_vec.py:140), so a backend keeps the settings it was built with.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Mapping


@dataclass(frozen=True)
class DebugTraps:
    trap_pc: int = 0
    trap_rst38: int = 0
    max_instr: int = 0
    watch_addr: int = 0

    @property
    def active(self) -> bool:
        return bool(self.trap_pc or self.trap_rst38 or self.max_instr or self.watch_addr)


def _parse(env: Mapping[str, str], name: str) -> int | None:
    text = env.get(name)
    if not text:
        return None
    try:
        return int(text, 0)
    except ValueError:
        return None


def read_debug_env(env: Mapping[str, str] | None = None) -> DebugTraps:
    """The four trap settings from ``env`` (default ``os.environ``)."""
    env = os.environ if env is None else env
    pc = _parse(env, "GBXCULE_TRAP_PC")
    mi = _parse(env, "GBXCULE_MAX_INSTR")
    wa = _parse(env, "GBXCULE_WATCH_ADDR")
    return DebugTraps(trap_pc=(pc & 0xFFFF) if pc is not None else 0,
                      trap_rst38=1 if env.get("GBXCULE_TRAP_RST38") else 0,
                      max_instr=max(0, mi) if mi is not None else 0,
                      watch_addr=(wa & 0xFFFF) if wa is not None else 0)
