"""Canonical per-env state schema in the reference's (env-major) layout.

The device keeps its own layout (see ``csrc/gbx_layout.h``); every parity
check converts to this schema, which lists the fields of the reference
backend's device buffers (``src/gbxcule/backends/warp_vec.py:279-497``) in one
fixed order so two implementations can be compared array by array or by a
single digest.
"""

from __future__ import annotations

import hashlib

import numpy as np

MEM_SIZE = 65536
SERIAL_MAX = 1024
SCREEN_H = 144
OBS_DIM = 32

# (name, dtype) per-env scalar fields, reference names.
SCALARS = (
    ("pc", np.int32), ("sp", np.int32), ("a", np.int32), ("b", np.int32),
    ("c", np.int32), ("d", np.int32), ("e", np.int32), ("h", np.int32),
    ("l", np.int32), ("f", np.int32),
    ("instr_count", np.int64), ("cycle_count", np.int64),
    ("cycle_in_frame", np.int32), ("trap_flag", np.int32), ("trap_pc", np.int32),
    ("trap_opcode", np.int32), ("trap_kind", np.int32),
    ("joyp_select", np.uint8), ("serial_len", np.int32), ("serial_overflow", np.uint8),
    ("ime", np.int32), ("ime_delay", np.int32), ("halted", np.int32),
    ("div_counter", np.int32), ("timer_prev_in", np.int32),
    ("tima_reload_pending", np.int32), ("tima_reload_delay", np.int32),
    ("ppu_scanline_cycle", np.int32), ("ppu_ly", np.int32), ("ppu_window_line", np.int32),
    ("ppu_stat_prev", np.uint8),
)
SCALAR_NAMES = tuple(n for n, _ in SCALARS)

# env-0 scanline latches (u8[144] each), reference order.
LATCHES = ("bg_lcdc", "bg_scx", "bg_scy", "bg_bgp", "win_wx", "win_wy",
           "win_line", "obj_obp0", "obj_obp1")

# Reference backend attribute names for each canonical field.
REF_ATTR = {n: "_" + n for n in SCALAR_NAMES}
REF_ATTR["l"] = "_l"
REF_ATTR.update({f"latch_{k}": f"_{k}_latch_env0" for k in LATCHES})
REF_ATTR.update({"mem": "_mem", "cart_state": "_cart_state", "cart_ram": "_cart_ram",
                 "serial_buf": "_serial_buf", "obs": "_obs", "reward": "_reward"})

ORDER = (("mem", "cart_ram", "cart_state") + SCALAR_NAMES + ("serial_buf",)
         + tuple(f"latch_{k}" for k in LATCHES) + ("obs", "reward"))


def digest(state: dict, fields=ORDER) -> str:
    """sha256 over the listed fields, each as little-endian contiguous bytes."""
    h = hashlib.sha256()
    for name in fields:
        arr = np.ascontiguousarray(np.asarray(state[name]).reshape(-1))
        h.update(name.encode())
        h.update(arr.astype(arr.dtype.newbyteorder("<"), copy=False).tobytes())
    return h.hexdigest()


def diff(a: dict, b: dict, num_envs: int, fields=ORDER, limit: int = 8) -> list[str]:
    """Human-readable list of the first mismatches between two states."""
    out = []
    for name in fields:
        x = np.asarray(a[name]).reshape(-1)
        y = np.asarray(b[name]).reshape(-1)
        if x.shape != y.shape:
            out.append(f"{name}: shape {x.shape} != {y.shape}")
            continue
        bad = np.nonzero(x != y)[0]
        if bad.size:
            per = max(1, x.size // max(1, num_envs)) if name not in ("obs",) else OBS_DIM
            k = int(bad[0])
            out.append(f"{name}: {bad.size} diffs, first flat={k} (env {k // per}, off {k % per}) "
                       f"{x[k]} != {y[k]}")
        if len(out) >= limit:
            break
    return out
