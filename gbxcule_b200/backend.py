"""The vectorized backend: drop-in for the reference's ``WarpVecCudaBackend``.

Same constructor keywords, attributes, methods, return types and error
messages as ``src/gbxcule/backends/warp_vec.py:86-1482`` of bkase/gbxcule, so
the reference's RL wrappers run unchanged apart from the import. Every device
operation goes through libgbx (``_lib.py``); there is no CPU path. Work is
enqueued on ``torch.cuda.current_stream()`` and host readbacks synchronise, as
in the reference.

Differences, all deliberate:
* ``boot_rom`` keyword (bytes or path). The reference reads
  ``bench/roms/bootrom_fast_dmg.bin`` relative to the working directory
  (``warp_vec.py:82,238-247``); the default here is the from-source stub of
  ``gbxcule_b200.roms.boot_stub``.
* ``device`` keyword selects the CUDA ordinal (the reference hard-codes
  ``cuda:0``), so one process per GPU can own its env slice.
* ``export_state``/``import_state`` give the full state in the reference's
  env-major layout (parity tooling, savestates).
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np

from . import _lib as L
from . import cartridge as cart
from .debug_traps import read_debug_env
from .roms import boot_stub
from .state import LATCHES, MEM_SIZE, OBS_DIM, SCALARS, SERIAL_MAX

DOWNSAMPLE_H, DOWNSAMPLE_W, DOWNSAMPLE_W_BYTES = 72, 80, 20
ROM_LIMIT = 0x8000

# action codec (src/gbxcule/core/action_codec.py:81-124)
ACTION_CODECS = {"pokemonred_puffer_v1": ("NOOP", "A", "B", "START", "UP", "DOWN", "LEFT", "RIGHT")}
DEFAULT_ACTION_CODEC_ID = "pokemonred_puffer_v1"


@dataclass(frozen=True)
class ArraySpec:
    """Shape/dtype/meaning of an array (backends/common.py:35-58)."""
    shape: tuple
    dtype: str
    meaning: str


def flags_from_f(f: int) -> dict:
    return {"z": (f >> 7) & 1, "n": (f >> 6) & 1, "h": (f >> 5) & 1, "c": (f >> 4) & 1}


class GbxVecCudaBackend:
    """Vectorized Game Boy envs on one B200, stepped by libgbx."""

    name: str = "gbx_vec_cuda"

    def __init__(
        self,
        rom_path: str | bytes,
        *,
        num_envs: int = 1,
        frames_per_step: int = 24,
        release_after_frames: int = 8,
        obs_dim: int = 32,
        base_seed: int | None = None,
        action_codec: str = DEFAULT_ACTION_CODEC_ID,
        stage: str = "obs_only",
        render_bg: bool = False,
        render_pixels: bool = False,
        render_pixels_packed: bool = False,
        render_on_step: bool = True,
        force_lcdc_on_render: bool = False,
        device: str | int = "cuda:0",
        boot_rom: bytes | str | None = None,
    ) -> None:
        if obs_dim != OBS_DIM:
            raise ValueError(f"obs_dim {obs_dim} unsupported; expected {OBS_DIM}")
        if stage not in L.STAGES:
            raise ValueError(f"unknown stage {stage!r}")
        if action_codec not in ACTION_CODECS:
            raise ValueError(f"Unknown action codec: {action_codec}")
        self.num_envs = int(num_envs)
        if self.num_envs <= 0:
            raise ValueError(f"num_envs must be > 0, got {num_envs}")
        self._rom_path = rom_path
        self._boot_src = boot_rom
        self._frames_per_step = int(frames_per_step)
        self._release_after_frames = int(release_after_frames)
        self._base_seed = base_seed
        self._stage = stage
        self._render_bg = bool(render_bg)
        self._render_pixels = bool(render_pixels)
        self._render_pixels_packed = bool(render_pixels_packed)
        self._render_on_step = bool(render_on_step)
        self._force_lcdc_on_render = bool(force_lcdc_on_render)
        # GBXCULE_TRAP_* / _MAX_INSTR / _WATCH_ADDR, read when the backend is
        # built, as the reference does when it fetches its kernel (warp_vec.py:140)
        self._debug = read_debug_env()
        self.action_codec = action_codec
        self.num_actions = len(ACTION_CODECS[action_codec])
        self.device = "cuda"
        self._ordinal = int(str(device).split(":")[-1]) if str(device) != "cuda" else 0
        self._libh = None  # libgbx, loaded by the first reset() (building needs nvcc)
        self._generation = 0  # bumped by reset() and close(); ResetCache checks it
        self._h = None
        self._initialized = False
        self._views: dict[str, Any] = {}
        self._rom_bytes: bytes | None = None
        self._bootrom_bytes: bytes | None = None
        self.action_spec = ArraySpec((self.num_envs,), "int32", f"action index [0, {self.num_actions})")
        self.obs_spec = ArraySpec((self.num_envs, obs_dim), "float32", "Observation vector per environment")

    # ------------------------------------------------------------------ helpers
    @property
    def _lib(self):
        if self._libh is None:
            self._libh = L.lib()
        return self._libh

    def _torch(self):
        import torch

        return torch

    def _stream(self):
        torch = self._torch()
        with torch.cuda.device(self._ordinal):
            return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def _need(self):
        if not self._initialized or self._h is None:
            raise RuntimeError("Backend not initialized. Call reset() first.")

    def _view(self, which: str):
        v = self._views.get(which)
        if v is None:
            v = L.torch_view(self._h, which)
            self._views[which] = v
        return v

    def _load_rom(self) -> bytes:
        src = self._rom_path
        if isinstance(src, (bytes, bytearray)):
            return bytes(src)
        p = Path(src)
        if not p.exists():
            raise FileNotFoundError(f"ROM file not found: {p}")
        return p.read_bytes()

    def _load_boot(self) -> bytes:
        src = self._boot_src
        if src is None:
            return boot_stub()
        data = bytes(src) if isinstance(src, (bytes, bytearray)) else Path(src).read_bytes()
        if len(data) != 0x100:
            raise ValueError(f"Boot ROM must be 256 bytes, got {len(data)}")
        return data

    # ------------------------------------------------------------------ lifecycle
    def reset(self, seed: int | None = None) -> tuple[np.ndarray, dict[str, Any]]:
        """(Re)allocate and initialise every env (warp_vec.py:249-513); seed is ignored."""
        rom, spec = cart.load_rom(self._load_rom())
        boot = self._load_boot()
        self._free()
        cfg = L.Config(self.num_envs, self._ordinal, L.STAGES[self._stage],
                       int(self._render_pixels), int(self._render_pixels_packed))
        h = ctypes.c_void_p()
        rb = (ctypes.c_uint8 * len(rom)).from_buffer_copy(rom)
        bb = (ctypes.c_uint8 * 256).from_buffer_copy(boot)
        L.check(self._lib.gbx_create(ctypes.byref(cfg), rb, len(rom), bb, 256, ctypes.byref(h)), "gbx_create")
        self._h = h
        d = self._debug
        L.check(self._lib.gbx_set_debug_traps(h, d.trap_pc, d.trap_rst38, d.max_instr, d.watch_addr),
                "gbx_set_debug_traps")
        self._spec = spec
        self._rom_bytes, self._bootrom_bytes = rom, boot
        info = L.Info()
        L.check(self._lib.gbx_get_info(h, ctypes.byref(info)))
        self._info = info
        L.check(self._lib.gbx_reset(h, self._stream()), "gbx_reset")
        self._initialized = True
        obs = np.zeros((self.num_envs, OBS_DIM), dtype=np.float32)
        if self._stage in ("obs_only", "full_step"):
            obs = self._read_obs()
        return obs, {"seed": seed}

    def _free(self) -> None:
        # Views handed out earlier stay valid: each holds its own reference to
        # the old batch, whose memory is freed when the last of them goes.
        self._views.clear()
        if self._h is not None:
            self._lib.gbx_destroy(self._h)
            self._h = None
            self._generation += 1
        self._initialized = False

    def close(self) -> None:
        """Release every device buffer; idempotent (warp_vec.py:1076-1141)."""
        self._free()
        self._rom_bytes = None
        self._bootrom_bytes = None

    def __del__(self):
        try:
            self._free()
        except Exception:
            pass

    # ------------------------------------------------------------------ stepping
    def _actions_buffer(self):
        return self._view("i32")[L.I32_FIELDS.index("actions")]

    def _launch_step(self, actions_ptr: int, frames: int | None = None, release: int | None = None,
                     render: bool = True) -> None:
        frames = self._frames_per_step if frames is None else frames
        release = self._release_after_frames if release is None else release
        s = self._stream()
        L.check(self._lib.gbx_step(self._h, ctypes.c_void_p(actions_ptr), int(frames), int(release), s), "gbx_step")
        if render and self._render_bg:  # env-0 frame from the scanline latches (warp_vec.py:651-671)
            L.check(self._lib.gbx_render_bg_env0(self._h, None, s), "gbx_render_bg_env0")
        if render and self._render_on_step:
            self._launch_render_pixels()

    def step(self, actions) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray, dict]:
        """Host path (warp_vec.py:515-563): validate, H2D actions, step, D2H obs."""
        self._need()
        acts = np.asarray(actions)
        if acts.shape != (self.num_envs,):
            raise ValueError(f"actions must have shape ({self.num_envs},), got {acts.shape}")
        acts = acts.astype(np.int32, copy=False)
        bad = (acts < 0) | (acts >= self.num_actions)
        if np.any(bad):
            raise ValueError(f"Action {int(acts[bad][0])} out of range [0, {self.num_actions})")
        torch = self._torch()
        buf = self._actions_buffer()
        buf.copy_(torch.from_numpy(np.ascontiguousarray(acts)), non_blocking=False)
        self._launch_step(buf.data_ptr())
        if self._stage in ("obs_only", "full_step"):
            obs = self._read_obs()
        else:
            obs = np.zeros((self.num_envs, OBS_DIM), dtype=np.float32)
        z = np.zeros((self.num_envs,), dtype=np.bool_)
        return obs, np.zeros((self.num_envs,), dtype=np.float32), z, z.copy(), {}

    def step_torch(self, actions) -> None:
        """Device path (warp_vec.py:1234-1269): int32 CUDA [num_envs], no host sync."""
        if not self._initialized:
            raise RuntimeError("Backend not initialized. Call reset() first.")
        torch = self._torch()
        if not isinstance(actions, torch.Tensor):
            raise TypeError("actions must be a torch.Tensor")
        if actions.device.type != "cuda":
            raise ValueError("actions must be a CUDA tensor")
        if actions.ndim != 1 or int(actions.shape[0]) != self.num_envs:
            raise ValueError(f"actions must have shape ({self.num_envs},)")
        if actions.dtype is not torch.int32:
            raise ValueError("actions must have dtype torch.int32 (no implicit cast)")
        if not actions.is_contiguous():
            raise ValueError("actions must be contiguous")
        if os.environ.get("GBXCULE_VALIDATE_ACTIONS") == "1":
            invalid = (actions < 0) | (actions >= self.num_actions)
            if torch.any(invalid).item():
                raise ValueError("actions contain out-of-range values")
        self._launch_step(actions.data_ptr())

    def _read_obs(self) -> np.ndarray:
        self._torch().cuda.synchronize(self._ordinal)
        return self._view("obs").cpu().numpy().copy()

    # ------------------------------------------------------------------ rendering
    def _apply_lcdc_override(self) -> None:
        mem = self.memory_torch()
        mem[:, 0xFF40] |= 0x80

    def _launch_render_pixels(self) -> None:
        if not (self._render_pixels or self._render_pixels_packed):
            return
        self._need()
        if self._force_lcdc_on_render:
            self._apply_lcdc_override()
        s = self._stream()
        if self._render_pixels:
            L.check(self._lib.gbx_render_shades(self._h, None, s), "gbx_render_shades")
        if self._render_pixels_packed:
            L.check(self._lib.gbx_render_packed(self._h, None, 0, s), "gbx_render_packed")

    def render_pixels_snapshot(self) -> None:
        """Render downsampled pixels without stepping CPU state (warp_vec.py:727-732)."""
        if not self._initialized:
            raise RuntimeError("Backend not initialized. Call reset() first.")
        self._launch_render_pixels()

    def render_pixels_snapshot_torch(self) -> None:
        """Render on the current torch CUDA stream (warp_vec.py:1271-1291)."""
        if not self._initialized:
            raise RuntimeError("Backend not initialized. Call reset() first.")
        self._launch_render_pixels()

    def render_pixels_snapshot_packed_to_torch(self, out, base_offset_bytes: int = 0) -> None:
        """Render packed pixels into a caller tensor (warp_vec.py:1293-1352)."""
        if not self._initialized or self._h is None:
            raise RuntimeError("Backend not initialized. Call reset() first.")
        torch = self._torch()
        if not isinstance(out, torch.Tensor):
            raise TypeError("out must be a torch.Tensor")
        if out.device.type != "cuda":
            raise ValueError("out must be a CUDA tensor")
        if out.dtype is not torch.uint8:
            raise ValueError("out must have dtype torch.uint8")
        if not out.is_contiguous():
            raise ValueError("out must be contiguous")
        if base_offset_bytes < 0:
            raise ValueError("base_offset_bytes must be >= 0")
        frame_bytes = self.num_envs * DOWNSAMPLE_W_BYTES * DOWNSAMPLE_H
        if base_offset_bytes + frame_bytes > int(out.numel()):
            raise ValueError("out does not have enough capacity for packed frame")
        if self._force_lcdc_on_render:
            self._apply_lcdc_override()
        L.check(self._lib.gbx_render_packed(self._h, ctypes.c_void_p(out.data_ptr()), int(base_offset_bytes),
                                            self._stream()), "gbx_render_packed")

    def render_pixels_snapshot_packed_scaled_to_torch(self, out, scaled, base_offset_bytes: int = 0,
                                                       layout: str = "rows") -> None:
        """``render_pixels_snapshot_packed_to_torch`` plus the policy input in
        the same launch: ``scaled`` (CUDA bf16, contiguous, >= N*72*80
        elements) receives every pixel as shade / 3.0 in bf16, the tensor a
        consumer gets from unpacking the packed bytes (rl/packed_pixels.py:26-71)
        and dividing by 3.0, as [N, 72, 80] rows (``layout="rows"``) or 2x2
        space-to-depth [N, 36, 40, 4] (``layout="s2d"``: pixel (y, x) at
        (y//2, x//2, (y%2)*2 + x%2)). ``out`` may be None (the backend's own
        packed buffer)."""
        if layout not in ("rows", "s2d"):
            raise ValueError(f"layout must be 'rows' or 's2d', got {layout!r}")
        if not self._initialized or self._h is None:
            raise RuntimeError("Backend not initialized. Call reset() first.")
        torch = self._torch()
        if not isinstance(scaled, torch.Tensor):
            raise TypeError("scaled must be a torch.Tensor")
        if scaled.device.type != "cuda" or scaled.dtype is not torch.bfloat16 or not scaled.is_contiguous():
            raise ValueError("scaled must be a contiguous CUDA bfloat16 tensor")
        if int(scaled.numel()) < self.num_envs * DOWNSAMPLE_H * DOWNSAMPLE_W_BYTES * 4:
            raise ValueError("scaled does not have enough capacity for the frames")
        ptr = None
        if out is not None:
            if not isinstance(out, torch.Tensor):
                raise TypeError("out must be a torch.Tensor")
            if out.device.type != "cuda" or out.dtype is not torch.uint8 or not out.is_contiguous():
                raise ValueError("out must be a contiguous CUDA uint8 tensor")
            if base_offset_bytes < 0:
                raise ValueError("base_offset_bytes must be >= 0")
            if base_offset_bytes + self.num_envs * DOWNSAMPLE_W_BYTES * DOWNSAMPLE_H > int(out.numel()):
                raise ValueError("out does not have enough capacity for packed frame")
            ptr = ctypes.c_void_p(out.data_ptr())
        if self._force_lcdc_on_render:
            self._apply_lcdc_override()
        L.check(self._lib.gbx_render_packed_scaled(self._h, ptr, int(base_offset_bytes),
                                                   ctypes.c_void_p(scaled.data_ptr()), int(layout == "s2d"),
                                                   self._stream()),
                "gbx_render_packed_scaled")

    def pixels_torch(self):
        """[N, 72, 80] uint8 view of the shade buffer (warp_vec.py:865-876)."""
        if self._h is None or not self._initialized or not self._render_pixels:
            raise RuntimeError("Pixel buffer not initialized. Call reset() first.")
        return self._view("pixels")

    def pixels_packed_torch(self):
        """[N, 72, 20] uint8 view of the packed buffer (warp_vec.py:887-901)."""
        if self._h is None or not self._initialized or not self._render_pixels_packed:
            raise RuntimeError("Packed pixel buffer not initialized. Call reset() first.")
        return self._view("pixels_packed")

    # ------------------------------------------------------------------ memory views / reads
    def memory_torch(self):
        """[N, 65536] uint8 zero-copy view of device memory (warp_vec.py:799-810).

        Device memory is env-major, so the view is contiguous like the
        reference's.
        """
        self._need()
        return self._view("mem")

    def read_memory_torch(self, env_idx: int, lo: int, hi: int):
        if env_idx < 0 or env_idx >= self.num_envs:
            raise ValueError(f"env_idx {env_idx} out of range [0, {self.num_envs})")
        if lo < 0 or hi < 0 or lo > MEM_SIZE or hi > MEM_SIZE or lo > hi:
            raise ValueError(f"Invalid memory range: lo={lo} hi={hi}")
        if lo < ROM_LIMIT:
            raise ValueError("read_memory_torch only supports RAM/IO ranges >= 0x8000")
        return self.memory_torch()[env_idx, lo:hi]

    def _read_rom_slice(self, lo: int, hi: int) -> bytes:
        """Unbanked ROM file bytes; the boot ROM below 0x100 (warp_vec.py:784-797)."""
        rom, boot = self._rom_bytes, self._bootrom_bytes
        out = bytearray(hi - lo)
        for k, addr in enumerate(range(lo, hi)):
            out[k] = boot[addr] if addr < 0x100 else (rom[addr] if addr < len(rom) else 0xFF)
        return bytes(out)

    def read_memory(self, env_idx: int, lo: int, hi: int) -> bytes:
        """Read [lo, hi) of one env (warp_vec.py:1354-1367)."""
        if self._h is None or not self._initialized:
            raise RuntimeError("Backend not initialized. Call reset() first.")
        if env_idx < 0 or env_idx >= self.num_envs:
            raise ValueError(f"env_idx {env_idx} out of range [0, {self.num_envs})")
        if lo < 0 or hi < 0 or lo > MEM_SIZE or hi > MEM_SIZE or lo > hi:
            raise ValueError(f"Invalid memory range: lo={lo} hi={hi}")
        if hi <= ROM_LIMIT:
            return self._read_rom_slice(lo, hi)
        mlo = max(lo, ROM_LIMIT)
        buf = (ctypes.c_uint8 * (hi - mlo))()
        L.check(self._lib.gbx_read_mem(self._h, env_idx, mlo, hi, buf), "gbx_read_mem")
        mem_part = bytes(buf)
        return (self._read_rom_slice(lo, ROM_LIMIT) if lo < ROM_LIMIT else b"") + mem_part

    def write_memory(self, env_idx: int, addr: int, data: bytes) -> None:
        raise NotImplementedError("CUDA write_memory is not implemented yet (debug-only for CPU).")

    # ------------------------------------------------------------------ state export
    def export_state(self, lo: int = 0, hi: int | None = None, *, parts=None) -> dict:
        """Full state of envs [lo, hi) in the reference's layout (``gbxcule_b200.state``)."""
        self._need()
        hi = self.num_envs if hi is None else hi
        n = hi - lo
        want = set(parts) if parts else {"mem", "cart_ram", "serial", "cart_state", "scalars", "latch",
                                         "obs", "reward"}
        ram_rows = max(self._info.ram_bytes, 1)
        mem = np.zeros((n, MEM_SIZE), np.uint8) if "mem" in want else None
        ram = np.zeros((n, ram_rows), np.uint8) if "cart_ram" in want else None
        ser = np.zeros((n, SERIAL_MAX), np.uint8) if "serial" in want else None
        cs = np.zeros((cart.CART_STATE_STRIDE, n), np.int32) if "cart_state" in want else None
        i32 = np.zeros((len(L.I32_FIELDS), n), np.int32) if "scalars" in want else None
        i64 = np.zeros((len(L.I64_FIELDS), n), np.int64) if "scalars" in want else None
        u8 = np.zeros((len(L.U8_FIELDS), n), np.uint8) if "scalars" in want else None
        lat = np.zeros((len(LATCHES), 144), np.uint8) if "latch" in want else None
        obs = np.zeros((n, OBS_DIM), np.float32) if "obs" in want else None
        rew = np.zeros((n,), np.float32) if "reward" in want else None

        def p(a):
            return None if a is None else a.ctypes.data_as(ctypes.c_void_p)

        hs = L.HostState(p(mem), p(ram), p(ser), p(cs), p(i32), p(i64), p(u8), p(lat), p(obs), p(rew))
        L.check(self._lib.gbx_export_state(self._h, lo, hi, ctypes.byref(hs)), "gbx_export_state")
        out: dict[str, Any] = {}
        if mem is not None:
            out["mem"] = mem.reshape(-1)
        if ram is not None:
            out["cart_ram"] = ram.reshape(-1)
        if ser is not None:
            out["serial_buf"] = ser.reshape(-1)
        if cs is not None:
            out["cart_state"] = np.ascontiguousarray(cs.T).reshape(-1)
        if i32 is not None:
            for k, name in enumerate(L.I32_FIELDS):
                out[name] = i32[k].copy()
            for k, name in enumerate(L.I64_FIELDS):
                out[name] = i64[k].copy()
            for k, name in enumerate(L.U8_FIELDS):
                out[name] = u8[k].copy()
        if lat is not None:
            for k, name in enumerate(LATCHES):
                out[f"latch_{name}"] = lat[k].copy()
        if obs is not None:
            out["obs"] = obs.reshape(-1)
        if rew is not None:
            out["reward"] = rew
        return out

    def import_state(self, state: dict, lo: int = 0, hi: int | None = None) -> None:
        """Write envs [lo, hi) from a dict in the ``export_state`` layout (missing keys skipped)."""
        self._need()
        hi = self.num_envs if hi is None else hi
        n = hi - lo
        keep = []

        def arr(key, shape, dtype, transpose=False):
            if key not in state:
                return None
            a = np.asarray(state[key], dtype=dtype).reshape(shape)
            a = np.ascontiguousarray(a.T if transpose else a)
            keep.append(a)
            return a.ctypes.data_as(ctypes.c_void_p)

        ram_rows = max(self._info.ram_bytes, 1)
        i32 = i64 = u8 = None
        if all(k in state for k in L.I32_FIELDS if k != "actions"):
            a = np.zeros((len(L.I32_FIELDS), n), np.int32)
            for k, name in enumerate(L.I32_FIELDS):
                if name in state:
                    a[k] = np.asarray(state[name]).reshape(n)
            keep.append(a)
            i32 = a.ctypes.data_as(ctypes.c_void_p)
            b = np.stack([np.asarray(state[k], np.int64).reshape(n) for k in L.I64_FIELDS])
            c = np.stack([np.asarray(state[k], np.uint8).reshape(n) for k in L.U8_FIELDS])
            keep.extend([b, c])
            i64, u8 = b.ctypes.data_as(ctypes.c_void_p), c.ctypes.data_as(ctypes.c_void_p)
        lat = None
        if all(f"latch_{k}" in state for k in LATCHES):
            la = np.stack([np.asarray(state[f"latch_{k}"], np.uint8) for k in LATCHES])
            keep.append(la)
            lat = la.ctypes.data_as(ctypes.c_void_p)
        hs = L.HostState(arr("mem", (n, MEM_SIZE), np.uint8), arr("cart_ram", (n, ram_rows), np.uint8),
                         arr("serial_buf", (n, SERIAL_MAX), np.uint8),
                         arr("cart_state", (n, cart.CART_STATE_STRIDE), np.int32, transpose=True),
                         i32, i64, u8, lat, arr("obs", (n, OBS_DIM), np.float32), arr("reward", (n,), np.float32))
        L.check(self._lib.gbx_import_state(self._h, lo, hi, ctypes.byref(hs)), "gbx_import_state")

    # ------------------------------------------------------------------ host reads (reference names)
    def get_cpu_state(self, env_idx: int) -> dict:
        """CPU registers and counters of one env (warp_vec.py:947-1009)."""
        if env_idx < 0 or env_idx >= self.num_envs:
            raise ValueError(f"env_idx {env_idx} out of range [0, {self.num_envs})")
        self._need()
        s = self.export_state(env_idx, env_idx + 1, parts=["scalars"])
        g = {k: int(v[0]) for k, v in s.items()}
        f = g["f"] & 0xF0
        return {"pc": g["pc"] & 0xFFFF, "sp": g["sp"] & 0xFFFF, "a": g["a"] & 0xFF, "f": f,
                "b": g["b"] & 0xFF, "c": g["c"] & 0xFF, "d": g["d"] & 0xFF, "e": g["e"] & 0xFF,
                "h": g["h"] & 0xFF, "l": g["l"] & 0xFF, "flags": flags_from_f(f),
                "instr_count": g["instr_count"], "cycle_count": g["cycle_count"],
                "trap_flag": g["trap_flag"], "trap_pc": g["trap_pc"] & 0xFFFF,
                "trap_opcode": g["trap_opcode"] & 0xFF, "trap_kind": g["trap_kind"]}

    def get_cart_state(self, env_idx: int) -> dict:
        """Cart/MBC record of one env (warp_vec.py:1435-1460)."""
        if env_idx < 0 or env_idx >= self.num_envs:
            raise ValueError(f"env_idx {env_idx} out of range [0, {self.num_envs})")
        self._need()
        cs = self.export_state(env_idx, env_idx + 1, parts=["cart_state"])["cart_state"]
        return {name: int(cs[k]) for k, name in enumerate(cart.CART_STATE_FIELDS)}

    def get_pc_snapshot(self) -> np.ndarray:
        self._need()
        self._torch().cuda.synchronize(self._ordinal)
        return self._view("i32")[0].cpu().numpy().copy()

    # ------------------------------------------------------------------ PyBoy state files
    def save_state(self, env_idx: int = 0):
        """Env ``env_idx`` as a ``PyBoyState`` (warp_vec.py:1024-1033)."""
        from .state_io import state_from_backend

        self._check_env(env_idx)
        return state_from_backend(self, env_idx)

    def save_state_file(self, path: str, env_idx: int = 0) -> None:
        """Write env ``env_idx`` as a PyBoy version-9 state file (warp_vec.py:1035-1044)."""
        from .state_io import save_pyboy_state

        save_pyboy_state(self.save_state(env_idx), path)

    def load_state(self, state, env_idx: int = 0) -> None:
        """Load a ``PyBoyState`` into env ``env_idx`` (warp_vec.py:1046-1055)."""
        from .state_io import apply_state_to_backend

        self._check_env(env_idx)
        apply_state_to_backend(state, self, env_idx)

    def load_state_file(self, path: str, env_idx: int = 0) -> None:
        """Load a PyBoy state file (versions 9-15) into env ``env_idx`` (warp_vec.py:1057-1074)."""
        from .state_io import load_pyboy_state

        self._need()
        state = load_pyboy_state(path, expected_cart_ram_size=int(self._spec.ram_byte_length))
        self.load_state(state, env_idx)

    def _check_env(self, env_idx: int) -> None:
        self._need()
        if env_idx < 0 or env_idx >= self.num_envs:
            raise ValueError(f"env_idx {env_idx} out of range [0, {self.num_envs})")

    def read_frame_bg_shade_env0(self) -> bytes:
        """Env 0's 160x144 frame, row-major, one shade per byte (warp_vec.py:1389-1404).

        Rendered after each step when the backend was built with
        ``render_bg=True``; zeros before the first such step.
        """
        self._need()
        self._torch().cuda.synchronize(self._ordinal)
        return self._view("frame_bg").cpu().numpy().tobytes()

    def read_serial(self, env_idx: int) -> bytes:
        if env_idx < 0 or env_idx >= self.num_envs:
            raise ValueError(f"env_idx {env_idx} out of range [0, {self.num_envs})")
        self._need()
        s = self.export_state(env_idx, env_idx + 1, parts=["serial", "scalars"])
        length = min(int(s["serial_len"][0]), SERIAL_MAX)
        return s["serial_buf"][:length].tobytes() if length > 0 else b""

    def drain_serial(self, env_idx: int) -> bytes:
        data = self.read_serial(env_idx)
        self._torch().cuda.synchronize(self._ordinal)
        self._view("i32")[L.I32_FIELDS.index("serial_len"), env_idx] = 0
        self._view("u8")[L.U8_FIELDS.index("serial_overflow"), env_idx] = 0
        return data

    def envs_per_warp(self) -> tuple[int, bool]:
        """(K of the latest step launch, whether K is settled) of the step kernel."""
        self._need()
        info = L.Info()
        L.check(self._lib.gbx_get_info(self._h, ctypes.byref(info)))
        return int(info.envs_per_warp), bool(info.envs_per_warp_tuned)

    def set_envs_per_warp(self, k: int) -> None:
        """Fix the step kernel's envs per warp (1..32), or 0 for the automatic choice."""
        self._need()
        L.check(self._lib.gbx_set_envs_per_warp(self._h, int(k)), "gbx_set_envs_per_warp")

    def dispatch(self) -> str:
        """Interpreter of the latest step launch: "switch" or "uniform"."""
        self._need()
        info = L.Info()
        L.check(self._lib.gbx_get_info(self._h, ctypes.byref(info)))
        return "uniform" if info.dispatch == L.DISPATCH["uniform"] else "switch"

    def set_dispatch(self, mode: str) -> None:
        """Fix the step kernel's interpreter ("switch" or "uniform"), or "auto"."""
        self._need()
        if mode not in L.DISPATCH:
            raise ValueError(f"dispatch must be one of {sorted(L.DISPATCH)}, got {mode!r}")
        L.check(self._lib.gbx_set_dispatch(self._h, L.DISPATCH[mode]), "gbx_set_dispatch")

    def device_status(self, clear: bool = False) -> int:
        """Device error bits (1: an env's mbc_kind differs from the cartridge)."""
        self._need()
        out = ctypes.c_uint32()
        L.check(self._lib.gbx_device_status(self._h, ctypes.byref(out), int(clear)))
        return int(out.value)


# Reference-compatible alias for code that imports the class by its old name.
WarpVecCudaBackend = GbxVecCudaBackend
