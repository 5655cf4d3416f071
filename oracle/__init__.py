"""CPU oracle for the emulator step (plain-C restatement of the reference).

TEST INFRASTRUCTURE: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline``/``--impl reference`` legs of ``bench.py`` may use this
package, and only as the checker or the CPU baseline. The product package
never imports it.

``OracleEnvs`` keeps state exactly in the reference backend's layout
(``src/gbxcule/backends/warp_vec.py:249-497``): env-major ``mem`` (64 KiB per
env), ``cart_state`` int32[20] per env, one array per scalar field. Its
``reset`` restates that initialisation (boot ROM copied to 0x0000-0x00FF,
bank_lo=1, bootrom_enabled=1, joyp_select=0x30, everything else zero) and,
for the ``obs_only``/``full_step`` stages, the zero-frame launch that fills
the observation buffer (``:498-512``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

from gbxcule_b200 import cartridge as cart
from gbxcule_b200.state import LATCHES, MEM_SIZE, OBS_DIM, SCALARS, SERIAL_MAX, SCREEN_H

HERE = Path(__file__).resolve().parent
SRC = HERE / "gbx_oracle.c"
LIB = HERE / "_build" / "libgbx_oracle.so"

STAGES = {"emulate_only": 0, "obs_only": 1, "reward_only": 2, "full_step": 3}


def build_oracle(force: bool = False) -> Path:
    """Compile the oracle with gcc (-O2, OpenMP, no fast-math)."""
    LIB.parent.mkdir(parents=True, exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-fno-fast-math",
               "-std=c11", "-Wall", "-o", str(LIB), str(SRC)]
        subprocess.run(cmd, check=True)
    return LIB


_P = ctypes.c_void_p


class _Ctx(ctypes.Structure):
    _fields_ = (
        [("rom", _P), ("bootrom", _P), ("rom_bank_count", ctypes.c_int32),
         ("rom_bank_mask", ctypes.c_int32), ("ram_bank_count", ctypes.c_int32),
         ("mem", _P), ("cart_ram", _P), ("cart_state", _P)]
        + [(n, _P) for n in ("pc", "sp", "a", "b", "c", "d", "e", "h", "l", "f",
                             "instr_count", "cycle_count", "cycle_in_frame", "trap_flag",
                             "trap_pc", "trap_opcode", "trap_kind", "actions", "joyp_select",
                             "serial_buf", "serial_len", "serial_overflow", "ime", "ime_delay",
                             "halted", "div_counter", "timer_prev_in", "tima_reload_pending",
                             "tima_reload_delay", "ppu_scanline_cycle", "ppu_ly",
                             "ppu_window_line", "ppu_stat_prev")]
        + [("latch", _P * 9), ("reward_out", _P), ("obs_out", _P),
           ("stage", ctypes.c_int32), ("num_envs", ctypes.c_int32), ("ram_ops", _P)]
    )


_lib = None


def _load():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build_oracle()))
        _lib.gbxo_step.argtypes = [ctypes.POINTER(_Ctx), ctypes.c_int32, ctypes.c_int32,
                                   ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]
        _lib.gbxo_render.argtypes = [_P, ctypes.c_int32, _P, ctypes.c_int32, ctypes.c_int32]
        _lib.gbxo_step_debug.argtypes = [ctypes.POINTER(_Ctx), ctypes.c_int32, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                         ctypes.POINTER(_Debug)]
        _lib.gbxo_render_bg_env0.argtypes = [_P, _P * 9, _P]
    return _lib


class _Debug(ctypes.Structure):
    _fields_ = [("trap_pc", ctypes.c_int32), ("trap_rst38", ctypes.c_int32),
                ("watch_addr", ctypes.c_int32), ("pad", ctypes.c_int32), ("max_instr", ctypes.c_int64)]


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


class OracleEnvs:
    """A batch of emulated consoles stepped by the C oracle."""

    def __init__(self, rom: bytes, boot: bytes, num_envs: int, *, stage: str = "obs_only",
                 threads: int | None = None, count_ram_ops: bool = False) -> None:
        self.rom, self.spec = cart.load_rom(rom)
        if len(boot) != 0x100:
            raise ValueError("boot ROM must be 256 bytes")
        self.boot = bytes(boot)
        self.num_envs = int(num_envs)
        self.stage = stage
        self.threads = threads or os.cpu_count() or 1
        # per-env RAM/IO bytes touched by the emulated instructions (gbx_oracle.c
        # gbxo_ctx.ram_ops), accumulated over every step when enabled
        self.ram_ops = np.zeros(self.num_envs, dtype=np.int64) if count_ram_ops else None
        from gbxcule_b200.debug_traps import read_debug_env

        # the reference reads its debug-trap variables when the backend is built
        self.debug = read_debug_env()
        self._lib = _load()
        self.reset()

    # -- state ---------------------------------------------------------------
    def reset(self) -> None:
        n, spec = self.num_envs, self.spec
        self.rom_np = np.frombuffer(self.rom, dtype=np.uint8).copy()
        self.boot_np = np.frombuffer(self.boot, dtype=np.uint8).copy()
        s = {}
        s["mem"] = np.zeros(n * MEM_SIZE, dtype=np.uint8)
        s["mem"].reshape(n, MEM_SIZE)[:, :0x100] = self.boot_np
        s["cart_ram"] = np.zeros(n * max(spec.ram_byte_length, 1), dtype=np.uint8)
        cs = np.zeros((n, cart.CART_STATE_STRIDE), dtype=np.int32)
        cs[:, cart.CS["mbc_kind"]] = spec.mbc_kind
        cs[:, cart.CS["rom_bank_lo"]] = 1
        cs[:, cart.CS["bootrom_enabled"]] = 1
        s["cart_state"] = cs.reshape(-1)
        for name, dt in SCALARS:
            s[name] = np.zeros(n, dtype=dt)
        s["joyp_select"][:] = 0x30
        s["serial_buf"] = np.zeros(n * SERIAL_MAX, dtype=np.uint8)
        for k in LATCHES:
            s[f"latch_{k}"] = np.zeros(SCREEN_H, dtype=np.uint8)
        s["obs"] = np.zeros(n * OBS_DIM, dtype=np.float32)
        s["reward"] = np.zeros(n, dtype=np.float32)
        s["actions"] = np.zeros(n, dtype=np.int32)
        self.s = s
        if self.stage in ("obs_only", "full_step"):
            self._run(0, 0)

    def _ctx(self) -> _Ctx:
        s, c = self.s, _Ctx()
        c.rom, c.bootrom = _ptr(self.rom_np), _ptr(self.boot_np)
        c.rom_bank_count = self.spec.rom_bank_count
        c.rom_bank_mask = self.spec.rom_bank_mask
        c.ram_bank_count = self.spec.ram_bank_count
        c.mem, c.cart_ram, c.cart_state = _ptr(s["mem"]), _ptr(s["cart_ram"]), _ptr(s["cart_state"])
        for name, _ in SCALARS:
            setattr(c, name, _ptr(s[name]))
        c.actions = _ptr(s["actions"])
        c.serial_buf = _ptr(s["serial_buf"])
        for k, nm in enumerate(LATCHES):
            c.latch[k] = _ptr(s[f"latch_{nm}"])
        c.reward_out, c.obs_out = _ptr(s["reward"]), _ptr(s["obs"])
        c.stage = STAGES[self.stage]
        c.num_envs = self.num_envs
        c.ram_ops = _ptr(self.ram_ops) if self.ram_ops is not None else None
        return c

    def _run(self, frames: int, release: int, lo: int = 0, hi: int | None = None) -> None:
        c = self._ctx()
        t = self.debug
        d = _Debug(trap_pc=t.trap_pc, trap_rst38=t.trap_rst38, watch_addr=t.watch_addr, pad=0,
                   max_instr=t.max_instr)
        self._lib.gbxo_step_debug(ctypes.byref(c), lo, self.num_envs if hi is None else hi,
                                  frames, release, self.threads, ctypes.byref(d))

    def step(self, actions: np.ndarray, frames: int = 24, release: int = 8) -> None:
        """One env-step for every env (``step_torch`` semantics: no range check)."""
        self.s["actions"][:] = np.asarray(actions, dtype=np.int32).reshape(-1)
        self._run(frames, release)

    # -- renderer ------------------------------------------------------------
    def render_packed(self) -> np.ndarray:
        out = np.zeros(self.num_envs * 1440, dtype=np.uint8)
        self._lib.gbxo_render(_ptr(self.s["mem"]), self.num_envs, _ptr(out), 1, self.threads)
        return out.reshape(self.num_envs, 72, 20)

    def render_bg_env0(self) -> np.ndarray:
        """Env 0's 160x144 BG frame from the scanline latches (ppu_step.py:11-176)."""
        out = np.zeros(144 * 160, dtype=np.uint8)
        lat = (_P * 9)(*[_ptr(self.s[f"latch_{k}"]) for k in LATCHES])
        self._lib.gbxo_render_bg_env0(_ptr(self.s["mem"]), lat, _ptr(out))
        return out

    def render_shades(self) -> np.ndarray:
        out = np.zeros(self.num_envs * 5760, dtype=np.uint8)
        self._lib.gbxo_render(_ptr(self.s["mem"]), self.num_envs, _ptr(out), 0, self.threads)
        return out.reshape(self.num_envs, 72, 80)

    # -- snapshot cache (core/reset_cache.py) ----------------------------------
    def snapshot(self, env_idx: int = 0) -> dict:
        """Capture env ``env_idx`` (the fields ResetCache.from_backend copies)."""
        s, n, e = self.s, self.num_envs, env_idx
        snap = {"mem": s["mem"].reshape(n, -1)[e].copy(),
                "cart_state": s["cart_state"].reshape(n, -1)[e].copy(),
                "cart_ram": s["cart_ram"].reshape(n, -1)[e].copy(),
                "serial_buf": s["serial_buf"].reshape(n, -1)[e].copy(),
                "actions": s["actions"][e].copy()}
        for name, _ in SCALARS:
            snap[name] = s[name][e].copy()
        return snap

    def restore(self, snap: dict, mask: np.ndarray) -> None:
        """Masked restore (``reset_cache.py:192-307``): only masked envs change."""
        s, n = self.s, self.num_envs
        m = np.asarray(mask).astype(bool).reshape(-1)
        for name in ("mem", "cart_state", "cart_ram", "serial_buf"):
            s[name].reshape(n, -1)[m] = snap[name]
        for name, _ in SCALARS:
            s[name][m] = snap[name]
        s["actions"][m] = snap["actions"]

    def state(self) -> dict:
        return self.s
