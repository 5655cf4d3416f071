"""Known-answer checks on the CUDA path, mirroring the reference's own unit
tests for this path (values poked through the zero-copy memory view, as the
reference's tests poke them with write_memory):

* scanline invariants and the VBlank request (tests/test_ppu_timing.py:28-58);
* env-0 scanline latches (tests/test_ppu_timing.py:61-89);
* synthetic tiles in the snapshot render (tests/test_ppu_downsampled_pixels.py:68-124);
* obs / reward formulas per stage, state untouched (tests/test_warp_vec_ws2_stage.py:60-154);
* masked restore including the shade image (tests/test_reset_cache.py:32-143);
* serial readback (tests/test_serial_output.py).
"""

from __future__ import annotations

import numpy as np
import pytest

from gbxcule_b200 import roms
from gbxcule_b200 import state as st
from oracle import OracleEnvs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _backend(rom, n, frames=1, **kw):
    from gbxcule_b200 import GbxVecCudaBackend

    be = GbxVecCudaBackend(rom, num_envs=n, frames_per_step=frames, release_after_frames=1, **kw)
    be.reset()
    return be


def _poke(be, o, env, addr, value):
    be.memory_torch()[env, addr] = value
    o.s["mem"].reshape(o.num_envs, -1)[env, addr] = value


def test_scanline_state_invariants_and_vblank_request():
    rom = roms.config1_rom()  # LCD off, no IO writes besides the joypad
    be = _backend(rom, 1)
    o = OracleEnvs(rom, roms.boot_stub(), 1)
    try:
        for addr, v in ((0xFFFF, 0x00), (0xFF0F, 0x00), (0xFF40, 0x80)):
            _poke(be, o, 0, addr, v)
        be.step_torch(torch.zeros(1, dtype=torch.int32, device="cuda"))
        o.step(np.zeros(1, np.int32), 1, 1)
        cpu = be.export_state()
        assert 0 <= int(cpu["ppu_ly"][0]) < 154
        assert 0 <= int(cpu["ppu_scanline_cycle"][0]) < 456
        assert be.read_memory(0, 0xFF0F, 0xFF10)[0] & 0x01 == 0x01
        assert not st.diff(cpu, o.state(), 1)
    finally:
        be.close()


def test_scanline_latch_captures_env0():
    rom = roms.config1_rom()
    be = _backend(rom, 2)
    o = OracleEnvs(rom, roms.boot_stub(), 2)
    try:
        for env in (0, 1):
            for addr, v in ((0xFF40, 0x91), (0xFF42, 0x22), (0xFF43, 0x11), (0xFF47, 0xE4)):
                _poke(be, o, env, addr, v)
        be.step_torch(torch.zeros(2, dtype=torch.int32, device="cuda"))
        o.step(np.zeros(2, np.int32), 1, 1)
        lat = be.export_state(parts=["latch"])
        assert int(lat["latch_bg_lcdc"][0]) == 0x91
        assert int(lat["latch_bg_scx"][0]) == 0x11
        assert int(lat["latch_bg_scy"][0]) == 0x22
        assert int(lat["latch_bg_bgp"][0]) == 0xE4
        assert not st.diff(be.export_state(), o.state(), 2)
    finally:
        be.close()


def test_synthetic_tiles_render_known_shades():
    rom = roms.config1_rom()
    be = _backend(rom, 2, render_pixels=True, render_pixels_packed=True, render_on_step=False)
    try:
        mem = be.memory_torch()
        mem[0, 0x8000:0x8010] = 0x00                  # colour 0 everywhere
        mem[1, 0x8000:0x8010] = 0xFF                  # colour 3 everywhere
        mem[:, 0x9800:0x9C00] = 0x00                  # map: tile 0
        mem[:, 0xFF47] = 0xE4                         # BGP: colour c -> shade c
        mem[:, 0xFF40] = 0x91                         # LCD, BG, tiles at 8000, map 9800
        be.render_pixels_snapshot_torch()
        torch.cuda.synchronize()
        pix = be.pixels_torch().cpu().numpy()
        assert (pix[0] == 0).all() and (pix[1] == 3).all()
        packed = be.pixels_packed_torch().cpu().numpy()
        assert (packed[0] == 0).all() and (packed[1] == 0xFF).all()
    finally:
        be.close()


@pytest.mark.parametrize("stage", ["obs_only", "reward_only", "full_step"])
def test_obs_and_reward_formulas(stage):
    rom = roms.config1_rom()
    n = 3
    be = _backend(rom, n, frames=0, stage=stage)
    try:
        rng = np.random.default_rng(4)
        s = be.export_state()
        regs = {"pc": rng.integers(0, 0x10000, n), "sp": rng.integers(0, 0x10000, n)}
        for r in ("a", "b", "c", "d", "e", "h", "l"):
            regs[r] = rng.integers(0, 256, n)
        regs["f"] = rng.integers(0, 16, n) << 4
        for k, v in regs.items():
            s[k] = v.astype(np.int32)
        wram = rng.integers(0, 256, (n, 16), dtype=np.uint8)
        s["mem"].reshape(n, -1)[:, 0xC000:0xC010] = wram
        be.import_state(s)
        before = be.export_state()
        be.step_torch(torch.zeros(n, dtype=torch.int32, device="cuda"))
        after = be.export_state()
        for k in st.ORDER:  # the stage writes obs/reward only
            if k not in ("obs", "reward", "instr_count", "cycle_count"):
                assert np.array_equal(np.asarray(before[k]), np.asarray(after[k])), k
        m = wram.astype(np.int64)
        g = {k: v.astype(np.int64) for k, v in regs.items()}
        want_obs = np.stack([g["pc"] / 65535.0, g["sp"] / 65535.0, g["a"] / 255.0, g["f"] / 255.0,
                             g["b"] / 255.0, g["c"] / 255.0, g["d"] / 255.0, g["e"] / 255.0,
                             g["h"] / 255.0, g["l"] / 255.0]
                            + [m[:, k] / 255.0 for k in range(16)]
                            + [((m[:, 0] ^ m[:, 1]) & 0xFF) / 255.0, ((m[:, 2] + m[:, 3] * 5) & 0xFF) / 255.0,
                               ((m[:, 4] ^ g["a"]) & 0xFF) / 255.0, ((m[:, 5] + g["b"]) & 0xFF) / 255.0,
                               ((m[:, 6] ^ g["c"]) & 0xFF) / 255.0, ((m[:, 7] + g["d"]) & 0xFF) / 255.0],
                            axis=1).astype(np.float32)
        want_rew = (((g["a"] ^ ((m[:, 0] + m[:, 1] * 3) & 0xFF)) & 0xFF) / 255.0).astype(np.float32)
        obs = after["obs"].reshape(n, 32)
        if stage in ("obs_only", "full_step"):
            np.testing.assert_array_equal(obs, want_obs)  # same f32 divisions, no fast-math
        if stage in ("reward_only", "full_step"):
            np.testing.assert_array_equal(after["reward"], want_rew)
    finally:
        be.close()


def test_masked_restore_includes_shade_image():
    """ResetCache restores the 72x80 shade image of masked envs from the
    snapshot (reset_cache.py:111-112,237-244) and leaves the packed image."""
    from gbxcule_b200 import ResetCache

    rom = roms.config2_rom()
    n = 8
    be = _backend(rom, n, frames=24, render_pixels=True, render_pixels_packed=True, render_on_step=True)
    try:
        acts = lambda k: torch.as_tensor(roms.uniform_actions(np.random.default_rng(k), n), device="cuda")  # noqa: E731
        for k in range(6):
            be.step_torch(acts(k))
        cache = ResetCache.from_backend(be, env_idx=2)
        snap_pix = be.pixels_torch()[2].clone()
        snap_state = be.export_state(2, 3)
        be.step_torch(acts(99))
        before_pix = be.pixels_torch().clone()
        before_packed = be.pixels_packed_torch().clone()
        mask = torch.tensor([1, 0, 1, 0, 0, 1, 0, 1], dtype=torch.bool, device="cuda")
        cache.apply_mask_torch(mask)
        torch.cuda.synchronize()
        pix = be.pixels_torch()
        for e in range(n):
            want = snap_pix if mask[e] else before_pix[e]
            assert torch.equal(pix[e], want), e
        assert torch.equal(be.pixels_packed_torch(), before_packed)
        for e in range(n):
            if mask[e]:
                one = be.export_state(e, e + 1)
                assert np.array_equal(one["mem"], snap_state["mem"])
                assert np.array_equal(one["cart_state"], snap_state["cart_state"])
    finally:
        be.close()


def test_serial_readback_matches_oracle(micro_roms):
    rom = bytes(micro_roms["SERIAL_HELLO"])
    be = _backend(rom, 2, frames=24)
    o = OracleEnvs(rom, roms.boot_stub(), 2)
    try:
        for _ in range(3):
            be.step_torch(torch.zeros(2, dtype=torch.int32, device="cuda"))
            o.step(np.zeros(2, np.int32), 24, 1)
        n0 = int(o.s["serial_len"][0])
        want = bytes(o.s["serial_buf"].reshape(2, -1)[0, :n0])
        assert n0 > 0
        assert be.read_serial(0) == want
        assert be.drain_serial(0) == want
        assert be.read_serial(0) == b""
        assert int(be.export_state(0, 1)["serial_len"][0]) == 0
    finally:
        be.close()


def _ime_rom() -> bytes:
    """Every IME transition in a loop: EI and RETI with an interrupt pending
    and with none, EI with IME already set, IF writes with IME on and off."""
    from gbxcule_b200.roms import Asm, finalize_header

    a = Asm(0x8000)
    for v in range(0, 0x40, 8):
        a.org(v)
        a.db(0xC9)                        # RST vectors: RET
    a.org(0x40)
    a.db(0x04, 0xD9)                      # VBlank vector: INC B; RETI
    a.org(0x48)
    a.db(0x14, 0xD9)                      # STAT vector: INC D; RETI
    a.org(0x150)
    a.ld_rr("sp", 0xDFF0)
    a.ld_r_d8("a", 0x00)
    a.ldh_store(0x40)                     # LCD off: IF changes only by writes
    a.ld_r_d8("a", 0x03)
    a.ldh_store(0xFF)                     # IE = VBlank | STAT
    a.label("loop")
    a.ld_r_d8("a", 0x01)
    a.ldh_store(0x0F)                     # IF = VBlank, IME = 0: pending, not serviced
    a.db(0x00)                            # NOP
    a.db(0xFB)                            # EI: IME 0 -> 1 with VBlank pending
    a.db(0x00)
    a.db(0xFB)                            # EI with IME already set, nothing pending
    a.ld_r_d8("a", 0x02)
    a.ldh_store(0x0F)                     # IF = STAT with IME set: serviced next
    a.db(0x0C)                            # INC C
    a.db(0xF3)                            # DI
    a.ld_r_d8("a", 0x03)
    a.ldh_store(0x0F)                     # both pending, IME = 0
    a.call("sub")                         # RETI there: IME 0 -> 1 with both pending
    a.db(0x1C)                            # INC E
    a.db(0xF3)                            # DI
    a.call("sub")                         # RETI with nothing pending
    a.db(0xFB)                            # EI, nothing pending
    a.jp("loop")
    a.label("sub")
    a.db(0xD9)
    return finalize_header(bytearray(a.finish()), title="IMEMIX", cart_type=0, rom_code=0, ram_code=0)


def test_ime_transitions_match_oracle():
    """The exact tail after EI/RETI (taken only when IME goes 0 -> 1) and
    after IF/IE writes services interrupts exactly where the reference does."""
    rom = _ime_rom()
    n = 3
    be = _backend(rom, n, frames=3)
    o = OracleEnvs(rom, roms.boot_stub(), n)
    try:
        rng = np.random.default_rng(9)
        for _ in range(3):
            acts = roms.uniform_actions(rng, n, 9)
            be.step_torch(torch.as_tensor(acts, device="cuda"))
            o.step(acts, 3, 1)
            got = be.export_state()
            assert not st.diff(got, o.state(), n)
        assert int(got["b"][0]) > 0 and int(got["d"][0]) > 0  # both handlers ran
    finally:
        be.close()
