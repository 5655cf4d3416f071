"""The step kernel's decode pinned to the reference's opcode table (GPU).

The every-opcode probe batch of ``tests/isa_probe.py`` (527 envs, one
instruction each, then a trap) through libgbx, with both interpreters: each opcode's next PC, cycle
count and trap behaviour must equal ``src/gbxcule/core/isa_sm83.py``'s table,
and the whole batch's state must equal the reference's own digest
(``isa_probe`` golden case, also replayed in ``test_gpu_parity.py``).
"""

from __future__ import annotations

import numpy as np
import pytest

from tests import isa_probe

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("k,dispatch", [(1, "switch"), (32, "switch"), (32, "uniform"), (1, "uniform")])
def test_every_opcode_on_the_gpu(k, dispatch):
    from gbxcule_b200 import GbxVecCudaBackend

    rom = isa_probe.rom_image()
    n = len(isa_probe.probes())
    be = GbxVecCudaBackend(rom, num_envs=n, frames_per_step=1, release_after_frames=1)
    be.reset()
    try:
        be.set_envs_per_warp(k)
        be.set_dispatch(dispatch)
        be.import_state(isa_probe.initial_state(rom))
        be.step_torch(torch.zeros(n, dtype=torch.int32, device="cuda"))
        bad = isa_probe.check(be.export_state())
        assert not bad, "\n".join(bad[:20])
    finally:
        be.close()
