"""The SM83 decode pinned to the reference's opcode table (CPU, oracle).

``tests/isa_probe.py`` runs every unprefixed and CB-prefixed opcode once
(conditional jumps, calls and returns taken and not taken) and reads back
where each sent the PC and how many cycles it took; here the oracle's answers
must equal the lengths, cycle counts and unimplemented set of
``src/gbxcule/core/isa_sm83.py`` (exported to ``golden/isa_sm83.json``). The
same batch runs on the GPU in ``test_gpu_isa.py`` and, through the reference's
own kernel source, in the ``isa_probe`` golden case.
"""

from __future__ import annotations

import numpy as np

from gbxcule_b200 import roms
from oracle import OracleEnvs
from tests import isa_probe


def test_table_shape_and_trap_set():
    t = isa_probe.isa_table()
    assert len(t["unprefixed"]) == 256 and len(t["cb"]) == 256
    unimpl = {r["opcode"] for r in t["unprefixed"] if not r["implemented"]}
    # the reference traps on STOP and the 11 illegal opcodes; 0xCB is its prefix
    assert unimpl == set(roms.ILLEGAL) | {roms.STOP, roms.PREFIX_CB}
    assert all(r["implemented"] for r in t["cb"])


def test_every_opcode_on_the_oracle():
    rom = isa_probe.rom_image()
    n = len(isa_probe.probes())
    o = OracleEnvs(rom, roms.boot_stub(), n)
    for name, arr in isa_probe.initial_state(rom).items():
        o.s[name][:] = np.asarray(arr).reshape(o.s[name].shape)
    o.step(np.zeros(n, np.int32), 1, 1)
    bad = isa_probe.check(o.state())
    assert not bad, "\n".join(bad[:20])
