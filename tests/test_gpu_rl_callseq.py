"""The reference RL env's backend call sequence on this backend (GPU).

``PokeredPackedParcelEnv`` (src/gbxcule/rl/pokered_packed_parcel_env.py) is
the reference's own consumer of the vectorized backend. It drives
``WarpVecCudaBackend`` with exactly these calls:

* the constructor with ``obs_dim=32, render_pixels=False,
  render_pixels_packed=True, render_on_step=False`` and
  ``force_lcdc_on_render`` (:98-109), then ``num_actions`` (:113);
* ``reset(seed=...)`` (:165);
* ``render_pixels_snapshot_packed_to_torch(pixels, 0)`` into a
  ``[N, 1, 72, 20]`` uint8 CUDA tensor (:169-176, :384);
* ``ResetCache.from_backend(backend, env_idx=0)`` and
  ``apply_mask_torch`` with an all-ones uint8 mask (:195-200), later with
  the done mask;
* ``step_torch(actions)`` with int32 CUDA actions (:383);
* ``memory_torch()`` column slices for its detectors: the 320 event bytes at
  0xD747, map id 0xD35E, player y/x 0xD361/0xD362 (:387-391), the bag and
  dialogue bytes of ``pokered_parcel_detectors.py:15-35``.

The env itself needs the reference tree and a CUDA device in one process,
which this build's test machines never offer together (the tree is not on
the GPU machine), so this test makes the same calls in the same order on the
config-5 cartridge and checks every observable they return against the
oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

from gbxcule_b200 import roms
from oracle import OracleEnvs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

EVENTS_START, EVENTS_LENGTH = 0xD747, 320
COLUMNS = (0xD35E, 0xD361, 0xD362, 0xD31D, 0xCFBE, 0xCF94, 0xCC26)


@pytest.mark.parametrize("force_lcdc", [False, True])
def test_reference_env_call_sequence(force_lcdc):
    from gbxcule_b200 import ResetCache, WarpVecCudaBackend

    rom = roms.config5_rom()
    n = 64
    be = WarpVecCudaBackend(rom, num_envs=n, frames_per_step=24, release_after_frames=8, obs_dim=32,
                            render_pixels=False, render_pixels_packed=True, render_on_step=False,
                            force_lcdc_on_render=force_lcdc)
    o = OracleEnvs(rom, roms.boot_stub(), n)
    try:
        assert int(be.num_actions) > 0
        be.reset(seed=0)
        pixels = torch.empty((n, 1, 72, 20), dtype=torch.uint8, device="cuda")
        be.render_pixels_snapshot_packed_to_torch(pixels, 0)
        if force_lcdc:  # the override sets LCDC bit 7 in every env before rendering
            o.s["mem"].reshape(n, -1)[:, 0xFF40] |= 0x80
        assert np.array_equal(pixels[:, 0].cpu().numpy(), o.render_packed())
        cache = ResetCache.from_backend(be, env_idx=0)
        cache.apply_mask_torch(torch.ones((n,), device="cuda", dtype=torch.uint8))
        snap = o.snapshot(0)
        o.restore(snap, np.ones(n, dtype=np.uint8))
        rng = np.random.default_rng(77)
        for k in range(6):
            acts = torch.as_tensor(roms.uniform_actions(rng, n, 9), device="cuda")
            be.step_torch(acts)
            o.step(acts.cpu().numpy(), 24, 8)
            be.render_pixels_snapshot_packed_to_torch(pixels, 0)
            if force_lcdc:
                o.s["mem"].reshape(n, -1)[:, 0xFF40] |= 0x80
            want = o.render_packed()
            assert np.array_equal(pixels[:, 0].cpu().numpy(), want), f"pixels step {k}"
            mem = be.memory_torch()
            om = o.s["mem"].reshape(n, -1)
            events = mem[:, EVENTS_START:EVENTS_START + EVENTS_LENGTH]
            assert np.array_equal(events.cpu().numpy(), om[:, EVENTS_START:EVENTS_START + EVENTS_LENGTH])
            for a in COLUMNS:
                assert np.array_equal(mem[:, a].cpu().numpy(), om[:, a]), f"column {a:#06x} step {k}"
            if k % 2:  # episode ends: the env restores its done envs from the cache
                done = np.random.default_rng(900 + k).random(n) < 0.3
                cache.apply_mask_torch(torch.as_tensor(done.astype(np.uint8), device="cuda"))
                o.restore(snap, done.astype(np.uint8))
        torch.cuda.synchronize()
        from gbxcule_b200 import state as st
        assert not st.diff(be.export_state(), o.state(), n)
    finally:
        be.close()
