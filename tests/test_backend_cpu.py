"""Host-side behaviour of the backend that needs no GPU: argument checks made
when the backend is built, the reference's "not initialized" errors before
``reset()`` (src/gbxcule/backends/warp_vec.py:503-901), and an idempotent
``close()``. Nothing here touches a device or loads libgbx: ``reset()`` is
never called, and the library is loaded by the first ``reset()``."""

from __future__ import annotations

import re

import numpy as np
import pytest

from gbxcule_b200 import GbxVecCudaBackend, roms

NOT_INIT = re.escape("Backend not initialized. Call reset() first.")


@pytest.fixture(scope="module")
def rom():
    return roms.config1_rom()


@pytest.mark.parametrize("kw, message", [
    ({"obs_dim": 16}, "obs_dim 16 unsupported; expected 32"),
    ({"action_codec": "x"}, "Unknown action codec: x"),
    ({"stage": "bogus"}, "unknown stage 'bogus'"),
    ({"num_envs": 0}, "num_envs must be > 0, got 0"),
])
def test_constructor_rejects_bad_arguments(rom, kw, message):
    with pytest.raises(ValueError, match=message):
        GbxVecCudaBackend(rom, **kw)


def test_calls_before_reset_raise_the_reference_errors(rom, monkeypatch):
    from gbxcule_b200 import _lib

    def no_library():
        raise AssertionError("libgbx loaded before reset()")

    monkeypatch.setattr(_lib, "lib", no_library)  # no toolkit needed before reset()
    be = GbxVecCudaBackend(rom, num_envs=2, render_pixels=True, render_pixels_packed=True)
    try:
        for call in (lambda: be.step(np.zeros(2, np.int32)), lambda: be.get_cpu_state(0),
                     lambda: be.read_memory(0, 0xC000, 0xC010), be.memory_torch,
                     lambda: be.read_memory_torch(0, 0xC000, 0xC010), be.render_pixels_snapshot,
                     lambda: be.get_cart_state(0), be.get_pc_snapshot, lambda: be.read_serial(0),
                     be.read_frame_bg_shade_env0):
            with pytest.raises(RuntimeError, match=NOT_INIT):
                call()
        with pytest.raises(RuntimeError, match="Pixel buffer not initialized. Call reset"):
            be.pixels_torch()
        with pytest.raises(RuntimeError, match="Packed pixel buffer not initialized. Call reset"):
            be.pixels_packed_torch()
    finally:
        be.close()
    be.close()  # idempotent, as the reference's close() (warp_vec.py:1076-1141)
