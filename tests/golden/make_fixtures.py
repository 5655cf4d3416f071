"""Generate the golden vectors that pin the oracle to the reference.

TEST INFRASTRUCTURE. Run only where the reference tree is available:

    python tests/golden/make_fixtures.py --reference <path-to-gbxcule> [--jobs 8]

It drives the reference's own backend (``WarpVecCpuBackend``) through
``ref_harness`` on

* the five synthetic config ROMs of ``gbxcule_b200.roms`` (small env counts),
  including the packed/unpacked snapshot renders and, for the MBC3 cartridge,
  a golden snapshot after 600 warm-up frames and seeded masked restores
  through the reference's CUDA restore kernels (``reset_mask.py``);
* the reference's 23 micro-ROMs (``bench/roms/build_micro_rom.py``) with the
  frame/release settings of ``bench/roms/suite.yaml``.

and writes per-step sha256 digests of the full canonical state
(``gbxcule_b200.state.ORDER``) to ``fixtures.json``. The micro-ROM images are
stored in ``micro_roms.npz`` with the header logo bytes (0x0104-0x0133)
zeroed; nothing in the emulator reads them, and the digests are taken on the
stored images.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys
import tempfile
import time
from concurrent.futures import ProcessPoolExecutor
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(REPO / "tests"))

from gbxcule_b200 import roms  # noqa: E402
from gbxcule_b200 import state as st  # noqa: E402

MICRO = [  # (name, frames_per_step, release_after_frames) from suite.yaml
    ("ALU_LOOP", 24, 8), ("MEM_RWB", 24, 8), ("SERIAL_HELLO", 24, 8),
    ("DMA_OAM_COPY", 1, 1), ("TIMER_DIV_BASIC", 24, 8), ("TIMER_IRQ_HALT", 24, 8),
    ("EI_DELAY", 24, 8), ("JOY_DIVERGE_PERSIST", 24, 8), ("LOADS_BASIC", 24, 8),
    ("ALU_FLAGS", 24, 8), ("ALU16_SP", 24, 8), ("FLOW_STACK", 24, 8),
    ("CB_BITOPS", 24, 8), ("MBC1_SWITCH", 24, 8), ("MBC1_RAM", 24, 8),
    ("MBC3_SWITCH", 24, 8), ("MBC3_RAM", 24, 8), ("BG_STATIC", 1, 1),
    ("BG_SCROLL_ANIM", 1, 1), ("PPU_WINDOW", 1, 1), ("PPU_SPRITES", 1, 1),
    ("PPU_STAT_IRQ", 1, 1), ("BG_SCROLL_SIGNED", 1, 1),
]


LONG_STEPS = 100

# unit 200 of config 1's loop: an instruction start every env reaches in the first step
TRAP_PC_CONFIG1 = "0x0326"


def _sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def _ref_state(be) -> dict:
    return {k: getattr(be, v).numpy() for k, v in st.REF_ATTR.items()}


def _ref_load(be, state: dict) -> None:
    """Write a state dict (``export_state`` layout) into the reference backend's arrays."""
    import array

    for name, attr in st.REF_ATTR.items():
        if name not in state:
            continue
        dst = getattr(be, attr).data
        vals = np.asarray(state[name]).reshape(-1)
        if isinstance(dst, bytearray):
            dst[:] = vals.astype(np.uint8).tobytes()
        else:
            dst[:] = array.array(dst.typecode, vals.tolist())


def _setup(case: dict, be) -> None:
    """Per-env start state of a case that does not start from reset alone."""
    if case.get("setup") == "isa_probe":
        import isa_probe

        _ref_load(be, isa_probe.initial_state(isa_probe.rom_image()))


def _actions(kind: str, rng, n: int) -> np.ndarray:
    if kind == "uniform9":
        return roms.uniform_actions(rng, n, 9)
    if kind == "uniform8":
        return roms.uniform_actions(rng, n, 8)
    if kind == "bernoulli":
        return roms.bernoulli_actions(rng, n, 0.3)
    if kind == "striped":
        return (np.arange(n) % 8).astype(np.int32)
    raise ValueError(kind)


def run_case(args) -> dict:
    ref_root, case = args
    import ref_harness as rh

    tmp = Path(tempfile.mkdtemp(prefix="gbxfix_"))
    boot = tmp / "boot.bin"
    boot.write_bytes(roms.boot_stub())
    rom_bytes = bytes.fromhex(case.pop("_rom_hex")) if "_rom_hex" in case else None
    if rom_bytes is None and case["rom"]["kind"] == "isa_probe":
        import isa_probe

        rom_bytes = isa_probe.rom_image()
    if rom_bytes is None:
        rom_bytes = roms.CONFIG_ROMS[case["rom"]["id"]]()
    rom_path = tmp / "rom.gb"
    rom_path.write_bytes(rom_bytes)
    case["rom"]["sha256"] = _sha(rom_bytes)
    # debug-trap cases set the reference's GBXCULE_* variables for this case
    # only (pool workers are reused across cases); the reference reads them
    # when the backend fetches its kernel
    saved_env = {k: os.environ.get(k) for k in case.get("env", {})}
    try:
        return _run_case(ref_root, case, rom_bytes, rom_path, boot)
    finally:
        for k, v in saved_env.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def _run_case(ref_root, case, rom_bytes, rom_path, boot) -> dict:
    import ref_harness as rh

    ref = rh.load_reference(ref_root, boot)  # clears any GBXCULE_* variables
    os.environ.update(case.get("env", {}))
    n = case["num_envs"]
    render_bg = case.get("render_bg", False)
    be = ref.backend(str(rom_path), num_envs=n, frames_per_step=case["frames"],
                     release_after_frames=case["release"], stage=case["stage"],
                     render_bg=render_bg)
    t0 = time.time()
    be.reset()
    case["reset_digest"] = st.digest(_ref_state(be))
    _setup(case, be)
    if "setup" in case:
        case["setup_digest"] = st.digest(_ref_state(be))
    rng = np.random.default_rng(case["action_seed"])
    steps = []
    render = case.get("render", False)
    draw = case.get("action_envs", n)  # actions drawn for this many envs; the first n are used

    def do_step():
        act = _actions(case["actions"], rng, draw)[:n]
        ref.launch_step(be, act, render=render_bg)
        rec = {"actions": act.tolist(), "digest": st.digest(_ref_state(be))}
        if render_bg:
            rec["frame_bg"] = _sha(ref.frame_bg(be).tobytes())
        if render:
            rec["render_packed"] = _sha(ref.render_packed(be).tobytes())
            rec["render_shades"] = _sha(ref.render_shades(be).tobytes())
        return rec

    for _ in range(case.get("warmup", 0)):
        rec = do_step()
        steps.append({"actions": rec["actions"], "digest": rec["digest"]})
    if "restore" in case:
        rs = case["restore"]
        cache = ref.reset_cache(be, env_idx=rs["snapshot_env"])
        ref.apply_mask_kernels(cache, np.ones(n, dtype=np.uint8))
        rs["after_full_restore"] = st.digest(_ref_state(be))
        mrng = np.random.default_rng(rs["mask_seed"])
        for _ in range(case["steps"]):
            rec = do_step()
            mask = (mrng.random(n) < rs["rate"]).astype(np.uint8)
            ref.apply_mask_kernels(cache, mask)
            rec["mask"] = mask.tolist()
            rec["after_restore"] = st.digest(_ref_state(be))
            steps.append(rec)
    else:
        for _ in range(case["steps"]):
            steps.append(do_step())
    case["trace"] = steps
    case["seconds"] = round(time.time() - t0, 1)
    return case


def _micro_roms(ref_root: Path) -> dict:
    src = ref_root / "bench" / "roms" / "build_micro_rom.py"
    sys.path.insert(0, str(ref_root / "src"))
    spec = importlib.util.spec_from_file_location("build_micro_rom", src)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = {}
    for name, _, _ in MICRO:
        rom = bytearray(getattr(mod, "build_" + name.lower())())
        rom[0x104:0x134] = bytes(0x30)
        out[name] = bytes(rom)
    return out


def cases(micro: dict) -> list[dict]:
    cs = [
        dict(name="config1", rom={"kind": "config", "id": 1}, num_envs=8, frames=24, release=8,
             stage="obs_only", actions="uniform9", action_seed=0, steps=4),
        dict(name="config1_f1", rom={"kind": "config", "id": 1}, num_envs=4, frames=1, release=1,
             stage="full_step", actions="uniform9", action_seed=10, steps=6),
        dict(name="config2", rom={"kind": "config", "id": 2}, num_envs=6, frames=24, release=8,
             stage="obs_only", actions="uniform9", action_seed=2, steps=4, render=True),
        dict(name="config3", rom={"kind": "config", "id": 3}, num_envs=8, frames=24, release=8,
             stage="obs_only", actions="bernoulli", action_seed=3, steps=4),
        dict(name="config4", rom={"kind": "config", "id": 4}, num_envs=6, frames=24, release=8,
             stage="obs_only", actions="uniform9", action_seed=4, steps=3, warmup=25,
             restore={"snapshot_env": 0, "rate": 0.34, "mask_seed": 1004}),
        dict(name="config5", rom={"kind": "config", "id": 5}, num_envs=4, frames=24, release=8,
             stage="obs_only", actions="uniform9", action_seed=5, steps=3, render=True),
    ]
    # env-0 160x144 BG frame from the scanline latches (render_bg=True)
    cs.append(dict(name="config2_bg", rom={"kind": "config", "id": 2}, num_envs=2, frames=24, release=8,
                   stage="obs_only", actions="uniform9", action_seed=21, steps=3, render_bg=True))
    cs.append(dict(name="micro_PPU_SPRITES_bg", rom={"kind": "micro", "id": "PPU_SPRITES"}, num_envs=2,
                   frames=1, release=1, stage="obs_only", actions="uniform8", action_seed=22, steps=3,
                   render_bg=True, _rom_hex=micro["PPU_SPRITES"].hex()))
    cs.append(dict(name="micro_PPU_WINDOW_bg", rom={"kind": "micro", "id": "PPU_WINDOW"}, num_envs=2,
                   frames=1, release=1, stage="obs_only", actions="uniform8", action_seed=23, steps=3,
                   render_bg=True, _rom_hex=micro["PPU_WINDOW"].hex()))
    # debug traps (GBXCULE_TRAP_PC / _TRAP_RST38 / _MAX_INSTR / _WATCH_ADDR)
    for name, cfg, env in [("trap_pc", 1, {"GBXCULE_TRAP_PC": TRAP_PC_CONFIG1}),
                           ("trap_rst38", 1, {"GBXCULE_TRAP_RST38": "1"}),
                           ("trap_max_instr", 2, {"GBXCULE_MAX_INSTR": "30000"}),
                           ("trap_watch", 1, {"GBXCULE_WATCH_ADDR": "0xDFEE"}),     # stack byte
                           ("trap_watch_div", 2, {"GBXCULE_WATCH_ADDR": "0xFF04"})]:  # DIV register
        cs.append(dict(name=name, rom={"kind": "config", "id": cfg}, num_envs=4, frames=24, release=8,
                       stage="obs_only", actions="uniform9", action_seed=30 + cfg, steps=3, env=env))
    # long horizons: 100 env-steps per config on 2 envs (configs 4 and 5 after the
    # 600-frame warm-up and a restore of every env from env 0, then seeded
    # masked restores each step). Config 1 uses the benchmark's own action
    # stream (default_rng(0) draws for 64 envs per step; envs 0-1 here).
    cs += [
        dict(name="config1_long", rom={"kind": "config", "id": 1}, num_envs=2, action_envs=64, frames=24,
             release=8, stage="obs_only", actions="uniform9", action_seed=0, steps=LONG_STEPS),
        dict(name="config2_long", rom={"kind": "config", "id": 2}, num_envs=2, frames=24, release=8,
             stage="obs_only", actions="uniform9", action_seed=12, steps=LONG_STEPS, render=True),
        dict(name="config3_long", rom={"kind": "config", "id": 3}, num_envs=2, frames=24, release=8,
             stage="obs_only", actions="bernoulli", action_seed=13, steps=LONG_STEPS),
        dict(name="config4_long", rom={"kind": "config", "id": 4}, num_envs=2, frames=24, release=8,
             stage="obs_only", actions="uniform9", action_seed=14, steps=LONG_STEPS, warmup=25,
             restore={"snapshot_env": 0, "rate": 0.1, "mask_seed": 1104}),
        dict(name="config5_long", rom={"kind": "config", "id": 5}, num_envs=2, frames=24, release=8,
             stage="obs_only", actions="uniform9", action_seed=15, steps=LONG_STEPS, warmup=25, render=True,
             restore={"snapshot_env": 0, "rate": 0.1, "mask_seed": 1105}),
    ]
    # every opcode once (conditionals taken and not taken), one env each, then a
    # trap: lengths, cycles and the trap set against the reference (tests/isa_probe.py)
    cs.append(dict(name="isa_probe", rom={"kind": "isa_probe"}, setup="isa_probe", num_envs=527, frames=1,
                   release=1, stage="obs_only", actions="uniform8", action_seed=40, steps=1))
    for name, frames, release in MICRO:
        steps = 3 if frames > 1 else 8
        cs.append(dict(name=f"micro_{name}", rom={"kind": "micro", "id": name}, num_envs=3,
                       frames=frames, release=release, stage="obs_only",
                       actions="striped" if name == "JOY_DIVERGE_PERSIST" else "uniform8",
                       action_seed=7, steps=steps, render=frames == 1,
                       _rom_hex=micro[name].hex()))
    return cs


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 1)
    ap.add_argument("--only", default=None, help="comma-separated case names")
    args = ap.parse_args()
    micro = _micro_roms(args.reference)
    np.savez_compressed(HERE / "micro_roms.npz",
                        **{k: np.frombuffer(v, dtype=np.uint8) for k, v in micro.items()})
    todo = cases(micro)
    if args.only:
        keep = set(args.only.split(","))
        todo = [c for c in todo if c["name"] in keep]
    with ProcessPoolExecutor(max_workers=args.jobs) as ex:
        done = list(ex.map(run_case, [(str(args.reference), c) for c in todo]))
    out_path = HERE / "fixtures.json"
    prev = json.loads(out_path.read_text())["cases"] if (args.only and out_path.exists()) else []
    by_name = {c["name"]: c for c in prev}
    for c in done:
        by_name[c["name"]] = c
        print(f"{c['name']}: {len(c['trace'])} steps in {c['seconds']}s")
    payload = {
        "about": "sha256 digests of the canonical state (gbxcule_b200.state.ORDER) after each "
                 "step, produced by running the reference's own backend and kernel source under "
                 "tests/golden/ref_harness.py",
        "cases": [by_name[k] for k in sorted(by_name)],
    }
    out_path.write_text(json.dumps(payload, indent=1) + "\n")


if __name__ == "__main__":
    main()
