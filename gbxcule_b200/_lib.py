"""ctypes binding of libgbx (include/gbx.h).

Loads the in-tree ``_build/libgbx.so`` (building it with nvcc if absent) and
raises if it cannot: there is no CPU or framework fallback for any entry point.
Status codes map to the reference backend's exception types: invalid argument
or range -> ``ValueError``, uninitialised/wrong state and CUDA failures ->
``RuntimeError``.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_int32, c_int64, c_size_t, c_uint32, c_void_p

GBX_OK, GBX_ERR_INVALID, GBX_ERR_CUDA, GBX_ERR_OOM, GBX_ERR_STATE, GBX_ERR_RANGE = range(6)
ABI_VERSION = 5  # include/gbx.h GBX_ABI_VERSION

BUF = {"mem": 0, "pixels": 1, "pixels_packed": 2, "obs": 3, "reward": 4, "cart_ram": 5,
       "serial": 6, "i32": 7, "i64": 8, "u8": 9, "cart_state": 10, "latch": 11, "frame_bg": 12}
I32_FIELDS = ("pc", "sp", "a", "b", "c", "d", "e", "h", "l", "f", "cycle_in_frame", "trap_flag",
              "trap_pc", "trap_opcode", "trap_kind", "serial_len", "ime", "ime_delay", "halted",
              "div_counter", "timer_prev_in", "tima_reload_pending", "tima_reload_delay",
              "ppu_scanline_cycle", "ppu_ly", "ppu_window_line", "actions")
I64_FIELDS = ("instr_count", "cycle_count")
U8_FIELDS = ("joyp_select", "serial_overflow", "ppu_stat_prev")
STAGES = {"emulate_only": 0, "obs_only": 1, "reward_only": 2, "full_step": 3}


class Config(ctypes.Structure):
    _fields_ = [("num_envs", c_int32), ("device", c_int32), ("stage", c_int32),
                ("alloc_pixels", c_int32), ("alloc_pixels_packed", c_int32)]


class Info(ctypes.Structure):
    _fields_ = [("num_envs", c_int32), ("env_stride", c_int32), ("device", c_int32), ("stage", c_int32),
                ("mbc_kind", c_int32), ("rom_bytes", c_int32), ("rom_bank_count", c_int32),
                ("rom_bank_mask", c_int32), ("ram_bank_count", c_int32), ("ram_bytes", c_int32),
                ("sm_count", c_int32), ("envs_per_warp", c_int32), ("envs_per_warp_tuned", c_int32),
                ("dispatch", c_int32)]


# gbx_dispatch (include/gbx.h)
DISPATCH = {"auto": 0, "switch": 1, "uniform": 2}


class BufferInfo(ctypes.Structure):
    _fields_ = [("data", c_void_p), ("dtype_code", c_int32), ("dtype_bits", c_int32), ("ndim", c_int32),
                ("shape", c_int64 * 3), ("strides", c_int64 * 3)]


class HostState(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("mem", "cart_ram", "serial", "cart_state", "i32", "i64", "u8s",
                                        "latch", "obs", "reward")]


_lib = None


def lib():
    """Load (and if needed build) libgbx; raises on any failure."""
    global _lib
    if _lib is not None:
        return _lib
    from . import build as _build

    path = _build.build()
    L = ctypes.CDLL(str(path))
    P, E = c_void_p, POINTER(c_void_p)
    sig = {
        "gbx_abi_version": ([], c_int32),
        "gbx_last_error": ([], c_char_p),
        "gbx_create": ([POINTER(Config), P, c_size_t, P, c_size_t, E], c_int32),
        "gbx_destroy": ([P], c_int32),
        "gbx_get_info": ([P, POINTER(Info)], c_int32),
        "gbx_reset": ([P, P], c_int32),
        "gbx_step": ([P, P, c_int32, c_int32, P], c_int32),
        "gbx_render_packed": ([P, P, c_int64, P], c_int32),
        "gbx_render_packed_scaled": ([P, P, c_int64, P, c_int32, P], c_int32),
        "gbx_render_shades": ([P, P, P], c_int32),
        "gbx_snapshot_create": ([P, c_int32, P, E], c_int32),
        "gbx_snapshot_destroy": ([P], c_int32),
        "gbx_masked_restore": ([P, P, P, P], c_int32),
        "gbx_buffer": ([P, c_int32, POINTER(BufferInfo)], c_int32),
        "gbx_export_dlpack": ([P, c_int32, E], c_int32),
        "gbx_export_state": ([P, c_int32, c_int32, POINTER(HostState)], c_int32),
        "gbx_import_state": ([P, c_int32, c_int32, POINTER(HostState)], c_int32),
        "gbx_read_mem": ([P, c_int32, c_int32, c_int32, P], c_int32),
        "gbx_device_status": ([P, POINTER(c_uint32), c_int32], c_int32),
        "gbx_render_bg_env0": ([P, P, P], c_int32),
        "gbx_set_debug_traps": ([P, c_int32, c_int32, c_int64, c_int32], c_int32),
        "gbx_set_envs_per_warp": ([P, c_int32], c_int32),
        "gbx_set_dispatch": ([P, c_int32], c_int32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    if L.gbx_abi_version() != ABI_VERSION:
        raise RuntimeError(f"libgbx ABI {L.gbx_abi_version()} != {ABI_VERSION}")
    _lib = L
    return L


def check(rc: int, what: str = "") -> None:
    if rc == GBX_OK:
        return
    msg = (lib().gbx_last_error() or b"").decode(errors="replace")
    if what:
        msg = f"{what}: {msg}"
    if rc in (GBX_ERR_INVALID, GBX_ERR_RANGE):
        raise ValueError(msg)
    raise RuntimeError(msg)


_pycapsule_new = ctypes.pythonapi.PyCapsule_New
_pycapsule_new.restype = ctypes.py_object
_pycapsule_new.argtypes = [c_void_p, c_char_p, c_void_p]


def torch_view(handle, which: str):
    """Zero-copy torch tensor over a device buffer, via a DLPack capsule."""
    import torch.utils.dlpack

    out = c_void_p()
    check(lib().gbx_export_dlpack(handle, BUF[which], ctypes.byref(out)), f"export {which}")
    cap = _pycapsule_new(out, b"dltensor", None)
    return torch.utils.dlpack.from_dlpack(cap)
