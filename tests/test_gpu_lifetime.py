"""Handle lifetime and launch-shape behaviour of the CUDA path on a B200.

* zero-copy views (DLPack) keep the batch they alias alive across ``reset()``
  and ``close()``, as the reference's ``wp.to_torch`` views keep their Warp
  arrays alive;
* a ``ResetCache`` taken before ``reset()`` is refused afterwards;
* the envs-per-warp choice of the step kernel changes no result, and the
  automatic choice settles on one of its candidates after its trial steps.
"""

from __future__ import annotations

import gc
import hashlib

import numpy as np
import pytest

from gbxcule_b200 import roms
from gbxcule_b200 import state as st

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _backend(rom, n, **kw):
    from gbxcule_b200 import GbxVecCudaBackend

    be = GbxVecCudaBackend(rom, num_envs=n, frames_per_step=24, release_after_frames=8, **kw)
    be.reset()
    return be


def _step(be, a):
    be.step_torch(torch.as_tensor(np.asarray(a, dtype=np.int32), device="cuda"))


def test_views_outlive_reset_and_close():
    rom = roms.config2_rom()
    n = 64
    be = _backend(rom, n, render_pixels_packed=True)
    rng = np.random.default_rng(7)
    for _ in range(2):
        _step(be, roms.uniform_actions(rng, n))
    be.render_pixels_snapshot_torch()
    mem, pix = be.memory_torch(), be.pixels_packed_torch()
    torch.cuda.synchronize()
    want_mem, want_pix = mem[:, 0x8000:].clone(), pix.clone()
    be.reset()  # a new batch; the old views still own the old one
    for _ in range(2):
        _step(be, roms.uniform_actions(rng, n))
    torch.cuda.synchronize()
    assert torch.equal(mem[:, 0x8000:], want_mem) and torch.equal(pix, want_pix)
    be.close()
    junk = torch.full((n, 65536), 0xA5, dtype=torch.uint8, device="cuda")  # reuse freed memory, if any
    torch.cuda.synchronize()
    assert torch.equal(mem[:, 0x8000:], want_mem) and torch.equal(pix, want_pix)
    mem[:, 0xC000] = 7  # the view is still writable memory of its own
    assert int(mem[3, 0xC000]) == 7
    del mem, pix, junk
    gc.collect()
    torch.cuda.synchronize()


def test_reset_cache_refused_after_reset():
    from gbxcule_b200 import ResetCache

    be = _backend(roms.config1_rom(), 8)
    try:
        cache = ResetCache.from_backend(be, env_idx=0)
        mask = torch.ones(8, dtype=torch.bool, device="cuda")
        cache.apply_mask_torch(mask)
        be.reset()
        with pytest.raises(RuntimeError, match="belongs to a backend that was reset or closed"):
            cache.apply_mask_torch(mask)
        cache.close()
    finally:
        be.close()


@pytest.mark.parametrize("cfg,n", [(2, 512), (4, 1024), (3, 2048)])
def test_envs_per_warp_changes_no_result(cfg, n):
    rom = roms.CONFIG_ROMS[cfg]()
    digests = {}
    for k, disp in ((1, "switch"), (4, "switch"), (32, "switch"), (32, "uniform"), (4, "uniform"), (0, "auto")):
        be = _backend(rom, n, render_pixels_packed=True)
        try:
            be.set_envs_per_warp(k)
            be.set_dispatch(disp)
            rng = np.random.default_rng(40 + cfg)
            for _ in range(7):
                _step(be, roms.bernoulli_actions(rng, n) if cfg == 3 else roms.uniform_actions(rng, n))
            be.render_pixels_snapshot_torch()
            torch.cuda.synchronize()
            pix = be.pixels_packed_torch().cpu().numpy().tobytes()
            digests[(k, disp)] = (st.digest(be.export_state()), hashlib.sha256(pix).hexdigest())
            used, settled = be.envs_per_warp()
            if k:
                assert used == k and settled and be.dispatch() == disp
            else:  # automatic: 6 trial steps (switch at K = 1 and 32, uniform at 32), then the fastest
                assert settled and used in (1, 32)
        finally:
            be.close()
    assert len(set(digests.values())) == 1, digests
