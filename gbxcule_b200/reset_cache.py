"""Snapshot-cache reset: drop-in for the reference's ``ResetCache``.

``from_backend`` captures one env into a device-resident snapshot and
``apply_mask_torch`` restores every masked env from it, on the current torch
stream, in a single libgbx launch (the reference issues ~37 Warp launches,
``src/gbxcule/core/reset_cache.py:192-307``). The restored fields are the
reference's: address space, cart state, cart RAM, serial buffer and every
per-env scalar; env-0 latches, obs and reward are left alone.
"""

from __future__ import annotations

import ctypes
from typing import Any

from . import _lib as L


class ResetCache:
    """Device snapshot of one env + masked restore (reset_cache.py:22-411)."""

    def __init__(self, backend: Any, snap: ctypes.c_void_p, env_idx: int) -> None:
        self.backend = backend
        self.num_envs = int(backend.num_envs)
        self.env_idx = env_idx
        self._snap = snap
        self._generation = backend._generation

    @classmethod
    def from_backend(cls, backend: Any, *, env_idx: int = 0) -> "ResetCache":
        """Capture env ``env_idx`` (reset_cache.py:67-190)."""
        if not getattr(backend, "_initialized", False):
            raise RuntimeError("Backend not initialized")
        out = ctypes.c_void_p()
        L.check(L.lib().gbx_snapshot_create(backend._h, int(env_idx), backend._stream(), ctypes.byref(out)),
                "gbx_snapshot_create")
        return cls(backend, out, int(env_idx))

    def apply_mask_torch(self, mask) -> None:
        """Restore envs where ``mask`` (bool/uint8 CUDA [num_envs]) is set (reset_cache.py:381-411)."""
        import torch

        backend = self.backend
        if backend.device != "cuda":
            raise RuntimeError("apply_mask_torch is only supported on CUDA backends.")
        if not isinstance(mask, torch.Tensor):
            raise TypeError("mask must be a torch.Tensor")
        if mask.device.type != "cuda":
            raise ValueError("mask must be a CUDA tensor")
        if mask.ndim != 1 or int(mask.shape[0]) != self.num_envs:
            raise ValueError(f"mask must have shape ({self.num_envs},)")
        if mask.dtype is torch.bool:
            mask_u8 = mask.to(torch.uint8)
        elif mask.dtype is torch.uint8:
            mask_u8 = mask
        else:
            raise ValueError("mask must be bool or uint8")
        mask_u8 = mask_u8.contiguous()
        if backend._h is None or backend._generation != self._generation:
            raise RuntimeError("ResetCache belongs to a backend that was reset or closed")
        L.check(L.lib().gbx_masked_restore(backend._h, self._snap, ctypes.c_void_p(mask_u8.data_ptr()),
                                           backend._stream()), "gbx_masked_restore")

    def apply_mask_np(self, mask) -> None:
        raise RuntimeError("apply_mask_np is only supported on CPU backends.")

    def close(self) -> None:
        if self._snap is not None and self._snap.value:
            L.lib().gbx_snapshot_destroy(self._snap)
        self._snap = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
