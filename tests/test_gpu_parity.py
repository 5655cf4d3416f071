"""Bit-exact parity of the CUDA path (libgbx via the backend) on a B200.

* every golden case (digests from the reference's own source) replayed through
  ``GbxVecCudaBackend`` / ``ResetCache``;
* CUDA vs the CPU oracle on the five config ROMs at larger env counts, full
  state every step;
* the benchmark-size configs (4,096 / 16,384 / 65,536 envs) with a seeded
  sample of envs replayed on the oracle from the same start state.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from gbxcule_b200 import roms
from gbxcule_b200 import state as st
from oracle import OracleEnvs
from tests.conftest import case_rom, case_setup_state

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def _cases():
    import json
    from tests.conftest import GOLDEN

    return json.loads((GOLDEN / "fixtures.json").read_text())["cases"]


def _backend(rom, n, frames, release, stage="obs_only", **kw):
    from gbxcule_b200 import GbxVecCudaBackend

    be = GbxVecCudaBackend(rom, num_envs=n, frames_per_step=frames, release_after_frames=release,
                           stage=stage, **kw)
    be.reset()
    return be


def _step(be, actions):
    be.step_torch(torch.as_tensor(np.asarray(actions, dtype=np.int32), device="cuda"))


# automatic launch shape (its trial steps include the uniform interpreter),
# and every step on the uniform interpreter at 32 envs per warp (a debug-trap
# case keeps its trap-checking switch instantiation either way)
@pytest.mark.parametrize("shape", ["auto", "uniform32"])
@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_golden_case_on_gpu(case, shape, micro_roms, monkeypatch):
    from gbxcule_b200 import ResetCache

    rom = case_rom(case, micro_roms)
    n = case["num_envs"]
    for k, v in case.get("env", {}).items():  # debug traps, read when the backend is built
        monkeypatch.setenv(k, v)
    be = _backend(rom, n, case["frames"], case["release"], case["stage"], render_pixels=True,
                  render_pixels_packed=True, render_on_step=False, render_bg=case.get("render_bg", False))
    if shape == "uniform32":
        be.set_envs_per_warp(32)
        be.set_dispatch("uniform")
    try:
        assert st.digest(be.export_state()) == case["reset_digest"]
        init = case_setup_state(case, rom)
        if init is not None:
            be.import_state(init)
            assert st.digest(be.export_state()) == case["setup_digest"]
        trace, warm = case["trace"], case.get("warmup", 0)
        for rec in trace[:warm]:
            _step(be, rec["actions"])
            assert st.digest(be.export_state()) == rec["digest"]
        cache = None
        if "restore" in case:
            rs = case["restore"]
            cache = ResetCache.from_backend(be, env_idx=rs["snapshot_env"])
            cache.apply_mask_torch(torch.ones(n, dtype=torch.bool, device="cuda"))
            assert st.digest(be.export_state()) == rs["after_full_restore"]
        for k, rec in enumerate(trace[warm:]):
            _step(be, rec["actions"])
            assert st.digest(be.export_state()) == rec["digest"], f"step {k}"
            if "frame_bg" in rec:
                assert _sha(be.read_frame_bg_shade_env0()) == rec["frame_bg"], f"env-0 frame step {k}"
            if "render_packed" in rec:
                be.render_pixels_snapshot_torch()
                torch.cuda.synchronize()
                assert _sha(be.pixels_packed_torch().cpu().numpy().tobytes()) == rec["render_packed"]
                assert _sha(be.pixels_torch().cpu().numpy().tobytes()) == rec["render_shades"]
            if "mask" in rec:
                cache.apply_mask_torch(torch.tensor(rec["mask"], dtype=torch.uint8, device="cuda"))
                assert st.digest(be.export_state()) == rec["after_restore"], f"restore step {k}"
    finally:
        be.close()


CONFIG_RUNS = [  # (config, envs, steps, frames, release, action kind)
    (1, 64, 6, 24, 8, "uniform9"),
    (2, 256, 6, 24, 8, "uniform9"),
    (3, 256, 5, 24, 8, "bernoulli"),
    (4, 128, 4, 24, 8, "uniform9"),
    (5, 64, 4, 24, 8, "uniform9"),
    (1, 37, 5, 3, 1, "uniform9"),     # ragged env count, short frames
]


def _acts(kind, rng, n):
    return roms.bernoulli_actions(rng, n) if kind == "bernoulli" else roms.uniform_actions(rng, n, 9)


# automatic mode runs its trial shapes (switch and uniform interpreters) on
# the first steps; the fixed shape holds the uniform interpreter throughout
@pytest.mark.parametrize("k,dispatch", [(0, "auto"), (32, "uniform")])
@pytest.mark.parametrize("cfg,n,steps,frames,release,kind", CONFIG_RUNS)
def test_cuda_matches_oracle(cfg, n, steps, frames, release, kind, k, dispatch):
    rom = roms.CONFIG_ROMS[cfg]()
    be = _backend(rom, n, frames, release, render_pixels_packed=True, render_on_step=True)
    be.set_envs_per_warp(k)
    be.set_dispatch(dispatch)
    o = OracleEnvs(rom, roms.boot_stub(), n)
    rng = np.random.default_rng(100 + cfg)
    try:
        for k in range(steps):
            a = _acts(kind, rng, n)
            _step(be, a)
            o.step(a, frames, release)
            d = st.diff(be.export_state(), o.state(), n)
            assert not d, f"config {cfg} step {k}: {d}"
            torch.cuda.synchronize()
            assert np.array_equal(be.pixels_packed_torch().cpu().numpy(), o.render_packed()), f"render step {k}"
    finally:
        be.close()


def _export_sample(be, sample):
    """Canonical state of the sampled envs, concatenated in sample order."""
    parts = [be.export_state(int(e), int(e) + 1) for e in sample]
    return {name: np.concatenate([np.asarray(p[name]).reshape(-1) for p in parts])
            for name in st.ORDER if not name.startswith("latch_")}


def _load_sample(be, o, sample):
    got = _export_sample(be, sample)
    for name, arr in got.items():
        o.s[name][:] = arr


FULL = [  # benchmark-size workloads: (config, envs, steps, action kind, restore rate)
    (2, 4096, 3, "uniform9", 0.0),
    (3, 16384, 2, "bernoulli", 0.0),
    (4, 65536, 2, "uniform9", 0.05),
    (5, 131072, 3, "uniform9", 0.05),
]


@pytest.mark.parametrize("cfg,n,steps,kind,rate", FULL)
def test_full_size_sampled_envs_match_oracle(cfg, n, steps, kind, rate):
    """Sampled envs of a full-size run replayed on the oracle, bit for bit."""
    from gbxcule_b200 import ResetCache

    rom = roms.CONFIG_ROMS[cfg]()
    be = _backend(rom, n, 24, 8, render_pixels_packed=True, render_on_step=True)
    rng = np.random.default_rng(1000 + cfg)
    sample = np.sort(rng.choice(n, size=24, replace=False))
    try:
        cache = None
        if rate > 0:
            # warm up, then restore everyone from env 0's snapshot (config 4 protocol)
            for _ in range(2):
                _step(be, _acts(kind, rng, n))
            cache = ResetCache.from_backend(be, env_idx=0)
            cache.apply_mask_torch(torch.ones(n, dtype=torch.bool, device="cuda"))
        o = OracleEnvs(rom, roms.boot_stub(), len(sample))
        _load_sample(be, o, sample)
        snap_o = o.snapshot(0)
        for k in range(steps):
            a = _acts(kind, rng, n)
            _step(be, a)  # render_on_step: the frames come from the state before the restore
            o.step(a[sample], 24, 8)
            want_pix = o.render_packed()
            if rate > 0:
                mask = (np.random.default_rng(2000 + k).random(n) < rate)
                cache.apply_mask_torch(torch.as_tensor(mask, device="cuda"))
                o.restore(snap_o, mask[sample].astype(np.uint8))
            got = _export_sample(be, sample)
            for name in st.ORDER:
                if name.startswith("latch_"):
                    continue
                assert np.array_equal(got[name], o.s[name]), f"config {cfg} step {k} field {name}"
            torch.cuda.synchronize()
            pix = be.pixels_packed_torch().cpu().numpy()[sample]
            assert np.array_equal(pix, want_pix), f"render step {k}"
    finally:
        be.close()


def test_config1_benchmark_size_every_step():
    """Config 1 as specified: 64 envs x 1,000 env-steps, the full state checked
    after every step against the oracle's committed per-step digests."""
    import json
    from tests.conftest import GOLDEN

    tr = json.loads((GOLDEN / "config1_1000.json").read_text())
    n = tr["envs"]
    be = _backend(roms.config1_rom(), n, tr["frames"], tr["release"])
    try:
        assert st.digest(be.export_state()) == tr["reset_digest"]
        rng = np.random.default_rng(tr["action_seed"])
        acts = torch.empty(n, dtype=torch.int32, device="cuda")
        for k, want in enumerate(tr["digests"]):
            acts.copy_(torch.from_numpy(roms.uniform_actions(rng, n, 9)))
            be.step_torch(acts)
            assert st.digest(be.export_state()) == want, f"step {k}"
    finally:
        be.close()


def test_determinism_and_zero_copy_views():
    """Two identical runs agree; torch views alias device state."""
    rom = roms.config2_rom()
    n = 512
    a = _backend(rom, n, 24, 8, render_pixels_packed=True)
    b = _backend(rom, n, 24, 8, render_pixels_packed=True)
    try:
        rng = np.random.default_rng(5)
        for _ in range(3):
            act = roms.uniform_actions(rng, n)
            _step(a, act)
            _step(b, act)
        assert st.digest(a.export_state()) == st.digest(b.export_state())
        mem = a.memory_torch()
        assert tuple(mem.shape) == (n, 65536)
        exp = a.export_state()["mem"].reshape(n, 65536)
        assert np.array_equal(mem[:, 0x8000:].cpu().numpy(), exp[:, 0x8000:])
        assert a.read_memory(3, 0xC000, 0xC010) == exp[3, 0xC000:0xC010].tobytes()
        assert a.read_memory(3, 0x0000, 0x0200)[:0x100] == roms.boot_stub()
        s = a.get_cpu_state(7)
        assert s["pc"] == int(a.export_state(7, 8)["pc"][0])
        assert a.device_status() == 0
        # writes through the view reach the device state
        mem[5, 0xC123] = 0xAB
        torch.cuda.synchronize()
        assert a.read_memory(5, 0xC123, 0xC124) == b"\xab"
    finally:
        a.close()
        b.close()


def test_api_errors_match_reference():
    from gbxcule_b200 import GbxVecCudaBackend, ResetCache

    rom = roms.config1_rom()
    be = GbxVecCudaBackend(rom, num_envs=8)
    with pytest.raises(RuntimeError, match="Call reset"):
        be.step_torch(torch.zeros(8, dtype=torch.int32, device="cuda"))
    be.reset()
    with pytest.raises(ValueError, match="out of range"):
        be.step(np.full(8, 9, dtype=np.int32))
    with pytest.raises(ValueError, match="int32"):
        be.step_torch(torch.zeros(8, dtype=torch.int64, device="cuda"))
    with pytest.raises(ValueError, match="shape"):
        be.step_torch(torch.zeros(7, dtype=torch.int32, device="cuda"))
    with pytest.raises(TypeError):
        be.step_torch(np.zeros(8, dtype=np.int32))
    with pytest.raises(ValueError, match="CUDA"):
        be.step_torch(torch.zeros(8, dtype=torch.int32))
    with pytest.raises(ValueError):
        be.get_cpu_state(8)
    with pytest.raises(ValueError, match="Invalid memory range"):
        be.read_memory(0, 10, 5)
    with pytest.raises(NotImplementedError):
        be.write_memory(0, 0xC000, b"\x00")
    out = torch.zeros(8 * 1440 - 1, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError, match="capacity"):
        be.render_pixels_snapshot_packed_to_torch(out)
    cache = ResetCache.from_backend(be)
    with pytest.raises(ValueError, match="bool or uint8"):
        cache.apply_mask_torch(torch.zeros(8, dtype=torch.int32, device="cuda"))
    obs, rew, done, trunc, info = be.step(np.zeros(8, dtype=np.int32))
    assert obs.shape == (8, 32) and obs.dtype == np.float32
    be.close()
    be.close()
    with pytest.raises(RuntimeError):
        be.memory_torch()


def test_render_into_offset_buffer_matches_oracle():
    rom = roms.config5_rom()
    n = 40
    be = _backend(rom, n, 24, 8)
    o = OracleEnvs(rom, roms.boot_stub(), n)
    rng = np.random.default_rng(9)
    try:
        for _ in range(3):
            a = roms.uniform_actions(rng, n)
            _step(be, a)
            o.step(a, 24, 8)
        for off in (0, 3, 16):
            out = torch.zeros(off + n * 1440 + 5, dtype=torch.uint8, device="cuda")
            be.render_pixels_snapshot_packed_to_torch(out, base_offset_bytes=off)
            torch.cuda.synchronize()
            got = out[off:off + n * 1440].cpu().numpy().reshape(n, 72, 20)
            assert np.array_equal(got, o.render_packed())
            assert int(out[:off].sum()) == 0 and int(out[off + n * 1440:].sum()) == 0
    finally:
        be.close()


def test_force_lcdc_on_render_matches_oracle():
    """force_lcdc_on_render sets LCDC bit 7 in every env's memory before the
    snapshot render (warp_vec.py:734-757); with the LCD switched off after the
    ROM filled VRAM, the render shows the tiles and later steps run with the
    LCD on, as in the reference."""
    rom = roms.config2_rom()
    n = 16
    be = _backend(rom, n, 24, 8, render_pixels_packed=True, render_on_step=True, force_lcdc_on_render=True)
    o = OracleEnvs(rom, roms.boot_stub(), n)
    rng = np.random.default_rng(77)
    try:
        for _ in range(6):  # the ROM's VRAM set-up
            a = roms.uniform_actions(rng, n)
            _step(be, a)
            o.step(a, 24, 8)
        be.memory_torch()[:, 0xFF40] &= 0x7F
        o.s["mem"].reshape(n, -1)[:, 0xFF40] &= 0x7F
        for k in range(2):
            a = roms.uniform_actions(rng, n)
            _step(be, a)
            o.step(a, 24, 8)
            o.s["mem"].reshape(n, -1)[:, 0xFF40] |= 0x80  # the override before the render
            torch.cuda.synchronize()
            assert not st.diff(be.export_state(), o.state(), n), f"step {k}"
            assert np.array_equal(be.pixels_packed_torch().cpu().numpy(), o.render_packed()), f"render {k}"
    finally:
        be.close()


@pytest.mark.parametrize("name", ["cfg2", "cfg4"])
def test_state_files_match_reference_on_gpu(name, tmp_path):
    """save_state_file writes the reference's bytes for the same state, and
    load_state_file puts a reference-saved file into an env exactly as the
    reference does (then stepping stays in parity)."""
    import json

    from tests.conftest import GOLDEN

    gold = json.loads((GOLDEN / "state_io.json").read_text())["cases"][name]
    blob = np.load(GOLDEN / "state_io.npz")[f"saved_{name}"].tobytes()
    rom = roms.CONFIG_ROMS[gold["config"]]()
    n = gold["num_envs"]
    be = _backend(rom, n, 24, 8)
    try:
        for a in gold["actions"]:
            _step(be, a)
        assert st.digest(be.export_state()) == gold["source_digest"]
        p = tmp_path / "s.state"
        be.save_state_file(str(p), env_idx=gold["env"])
        assert p.read_bytes() == blob
    finally:
        be.close()
    be = _backend(rom, n, 24, 8)
    try:
        p = tmp_path / "ref.state"
        p.write_bytes(blob)
        be.load_state_file(str(p), env_idx=0)
        assert st.digest(be.export_state()) == gold["applied_digest"]
        for rec in gold["after"]:
            _step(be, rec["actions"])
            assert st.digest(be.export_state()) == rec["digest"]
    finally:
        be.close()


def test_policy_rollout_with_resets_replays_on_oracle():
    """Config-5 rollout shape: packed frames (and the policy's bf16 input from
    the same render) -> bf16 policy -> sampled actions -> step_torch, with
    masked restores from a ResetCache; the recorded actions and masks
    replayed on the oracle give the same state and frames."""
    from gbxcule_b200 import ResetCache, rollout

    rom = roms.config5_rom()
    n = 48
    be = _backend(rom, n, 24, 8, render_pixels_packed=True, render_on_step=False)
    o = OracleEnvs(rom, roms.boot_stub(), n)
    try:
        a0 = roms.uniform_actions(np.random.default_rng(5), n)
        _step(be, a0)
        o.step(a0, 24, 8)
        cache = ResetCache.from_backend(be, env_idx=0)
        snap = o.snapshot(0)
        pol = rollout.make_policy("cuda")
        gen = torch.Generator(device="cuda").manual_seed(11)
        masks = [torch.as_tensor(np.random.default_rng(60 + k).random(n) < 0.25, device="cuda") for k in range(4)]
        frames = []
        orig = be.render_pixels_snapshot_packed_scaled_to_torch

        def rec(out, scaled, base_offset_bytes=0, layout="rows"):
            orig(out, scaled, base_offset_bytes, layout)
            frames.append(out.clone())
            # the policy's input: the packed frame unpacked, as bf16, / 3.0
            want = rollout.unpack_2bpp_u8(out).unsqueeze(1).to(torch.bfloat16) / 3.0
            if layout == "s2d":
                want = rollout.s2d_frames(want)
            assert torch.equal(scaled.view(torch.int16), want.reshape(scaled.shape).view(torch.int16))

        be.render_pixels_snapshot_packed_scaled_to_torch = rec
        ro = rollout.run_rollout(be, pol, 4, generator=gen, reset_cache=cache, reset_mask=lambda k: masks[k])
        for k in range(4):
            assert np.array_equal(frames[k].cpu().numpy(), o.render_packed()), f"policy input {k}"
            a = ro.actions[k].cpu().numpy()
            assert a.min() >= 0 and a.max() < 9
            o.step(a, 24, 8)
            o.restore(snap, masks[k].cpu().numpy().astype(np.uint8))
        assert not st.diff(be.export_state(), o.state(), n)
    finally:
        be.close()


def test_two_rank_slices_equal_one_batch():
    """Two handles on one GPU, each a rank's contiguous env slice stepped with
    its own action stream (multi.rank_seed), end in the states one batch of
    all the global env ids reaches with the same per-slice streams."""
    from gbxcule_b200 import multi

    rom, per, world, steps = roms.config5_rom(), 192, 2, 3
    whole = _backend(rom, per * world, 24, 8)
    parts = [_backend(rom, per, 24, 8) for _ in range(world)]
    rngs = [np.random.default_rng(multi.rank_seed(11, r)) for r in range(world)]
    try:
        for _ in range(steps):
            acts = [roms.uniform_actions(g, per, 9) for g in rngs]
            for be, a in zip(parts, acts):
                _step(be, a)
            _step(whole, np.concatenate(acts))
        full = whole.export_state()
        for r, be in enumerate(parts):
            lo, hi = multi.rank_env_slice(r, world, per)
            mine = be.export_state()
            for name in st.ORDER:
                if name.startswith("latch_"):  # env-0 latches belong to each batch's env 0
                    continue
                a = np.asarray(mine[name]).reshape(per, -1)
                b = np.asarray(full[name]).reshape(per * world, -1)[lo:hi]
                assert np.array_equal(a, b), f"rank {r} field {name}"
    finally:
        whole.close()
        for be in parts:
            be.close()


def test_scaled_render_equals_unpacked_frames_over_three():
    """gbx_render_packed_scaled: the packed bytes equal the plain packed
    render, and the bf16 image equals unpack -> bf16 -> / 3.0 bit for bit,
    at an offset into a larger packed buffer as well."""
    from gbxcule_b200 import rollout

    rom = roms.config2_rom()
    n = 48
    be = _backend(rom, n, 24, 8, render_pixels_packed=True)
    try:
        rng = np.random.default_rng(8)
        for _ in range(7):  # past the ROM's VRAM set-up: tiles, window and sprites on screen
            _step(be, roms.uniform_actions(rng, n))
        plain = torch.empty((n, 72, 20), dtype=torch.uint8, device="cuda")
        be.render_pixels_snapshot_packed_to_torch(plain)
        big = torch.zeros(1440 * n + 4096, dtype=torch.uint8, device="cuda")
        scaled = torch.full((n, 1, 72, 80), -1.0, dtype=torch.bfloat16, device="cuda")
        be.render_pixels_snapshot_packed_scaled_to_torch(big, scaled, 1024)
        torch.cuda.synchronize()
        assert torch.equal(big[1024:1024 + 1440 * n].view(n, 72, 20), plain)
        assert int(big[:1024].sum()) == 0 and int(big[1024 + 1440 * n:].sum()) == 0
        want = rollout.unpack_2bpp_u8(plain).unsqueeze(1).to(torch.bfloat16) / 3.0
        assert torch.equal(scaled.view(torch.int16), want.view(torch.int16))
        assert len(torch.unique(want)) > 1
        s2d = torch.empty((n, 36, 40, 4), dtype=torch.bfloat16, device="cuda")
        be.render_pixels_snapshot_packed_scaled_to_torch(None, s2d, layout="s2d")
        torch.cuda.synchronize()
        assert torch.equal(s2d.view(torch.int16), rollout.s2d_frames(want).view(torch.int16))
        assert torch.equal(be.pixels_packed_torch(), plain)
        with pytest.raises(ValueError):
            be.render_pixels_snapshot_packed_scaled_to_torch(None, scaled.float())
    finally:
        be.close()


def test_fused_policy_matches_module_within_bf16_tolerance():
    """The policy's GPU paths (each Conv2d + bias + ReLU as one cuDNN call;
    the first convolution also over the space-to-depth frame) against the
    plain module on the same bf16 input: equal up to bf16 rounding
    (tolerance: 2 % of the largest logit + 0.02)."""
    from gbxcule_b200 import rollout

    pol = rollout.make_policy("cuda", seed=3)
    g = torch.Generator(device="cuda").manual_seed(4)
    shades = torch.randint(0, 4, (512, 72, 80), generator=g, device="cuda", dtype=torch.uint8)
    with torch.no_grad():
        x = shades.unsqueeze(1).to(torch.bfloat16) / 3.0
        fused = pol.forward_scaled(x).float()
        plain = pol.head(pol.conv(x.contiguous(memory_format=torch.channels_last))).float()
        s2d = pol.forward_s2d(rollout.s2d_frames(x)).float()
    tol = 0.02 * float(plain.abs().max()) + 0.02
    assert float((fused - plain).abs().max()) <= tol
    assert float((s2d - plain).abs().max()) <= tol
