#!/usr/bin/env python
"""Benchmark: env-steps/s (frameskip 24) of the B200 Game Boy core.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl gbx|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

Workload (config 2 of the five benchmark configs): synthetic seeded ROM with the
PPU on (LCDC=0xE3), 4,096 envs per GPU, 24 frames per env-step, release after
8 frames, uniform actions from the 9-action codec (seed 0 + rank), and the
72x20 packed 2-bpp observation rendered every step. Envs are independent, so
N GPUs run N independent env slices (weak scaling, no collective on the step
path); ranks meet only for the barrier and the max-over-ranks timing.

Prints one JSON line on rank 0:
* value       env-steps/s of the whole job, inputs resident in HBM, step +
              render kernels timed with CUDA events per step (L2 flushed
              between timed steps), max over ranks;
* e2e         the same through the public API with host buffers: actions
              H2D from pinned memory and the packed frames D2H every step;
* roofline    the step kernel's algorithmic HBM bytes per launch / its mean
              event-timed duration vs the measured HBM peak (the kernel is
              integer-issue/latency bound; the issue counters are in profiles/);
* cpu_baseline the CPU oracle (C restatement of the reference step) on the
              host cores, on a bounded sample of the same workload.
``--impl reference`` times the reference's CPU implementation of the path;
the reference's Warp runtime cannot be installed here, so that arm runs the
oracle on all host threads over the same workload (kind "port").
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ENVS_PER_GPU = 4096
FRAMES = 24
RELEASE = 8
CONFIG = 2
METRIC = "env-steps/s (frameskip 24)"
UNIT = "env-steps/s"
WORKLOAD = "config2: PPU on (LCDC=0xE3) random-opcode loop, 4096 envs/GPU, frameskip 24, packed 72x20 obs"

# Algorithmic HBM bytes of one env-step of the step kernel (read + write of
# every per-env field it owns, the action, the f32 obs vector). Instruction
# RAM traffic is not counted, so this is a lower bound.
STEP_STATE_BYTES = 2 * (27 * 4 + 2 * 8 + 3 + 20 * 4 + 12) + 4 + 32 * 4
# dram__bytes_read.sum + dram__bytes_write.sum of one step-kernel launch on
# this workload (4,096 envs), from an ncu --set full capture of
# `bench.py --steps 3 --warmup 3 --no-cpu-baseline`. It includes the
# emulated programs' RAM lines and the write-back of the L2 flush buffer
# written just before the launch.
STEP_KERNEL_DRAM_BYTES_4096 = 64.935168e6 + 146.290944e6
# smsp__inst_executed.sum / emulated SM83 instructions of one step-kernel
# launch on this workload, from the same ncu capture: the integer-issue cost
# of one emulated instruction, used for the issue roofline below.
WARP_INSTR_PER_EMULATED_INSTR = 48.096002450e9 / (4096 * 197327.3)
SMS, ISSUE_PER_SM_PER_CLOCK = 148, 4


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _issue_roofline(emu_instr_per_s_per_gpu: float, clk: dict) -> dict:
    mhz = clk.get("sm_mhz") or 1965.0
    peak = SMS * ISSUE_PER_SM_PER_CLOCK * mhz * 1e6
    achieved = emu_instr_per_s_per_gpu * WARP_INSTR_PER_EMULATED_INSTR
    return {"bound": "integer issue", "achieved": achieved, "peak": peak, "unit": "warp-instructions/s per GPU",
            "frac": achieved / peak, "warp_instr_per_emulated_instr": WARP_INSTR_PER_EMULATED_INSTR,
            "note": "warp instructions per emulated instruction from an ncu capture of this workload"}


def _cpu_model() -> str:
    """Host CPU model name (Linux /proc/cpuinfo), recorded beside the CPU baseline."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_oracle_rate(total_envs_hint: int, warmup: int, steps: int, threads: int, seed: int = 0) -> dict:
    """Time the CPU oracle on a bounded sample of the workload (env-steps/s)."""
    from gbxcule_b200 import roms
    from oracle import OracleEnvs

    m = min(total_envs_hint, 48 * threads)
    rom = roms.CONFIG_ROMS[CONFIG]()
    o = OracleEnvs(rom, roms.boot_stub(), m, threads=threads)
    rng = np.random.default_rng(seed)
    for _ in range(warmup):
        o.step(roms.uniform_actions(rng, m, 9), FRAMES, RELEASE)
    t0 = time.perf_counter()
    for _ in range(steps):
        o.step(roms.uniform_actions(rng, m, 9), FRAMES, RELEASE)
        o.render_packed()
    dt = time.perf_counter() - t0
    return {"value": m * steps / dt, "unit": UNIT, "cores": threads, "kind": "port", "cpu_model": _cpu_model(),
            "sample": f"{m} envs x {steps} env-steps (after {warmup} warm-up steps) of the config-2 workload, "
                      f"oracle step + packed render, {threads} threads, {dt:.1f} s"}


def run_reference(args) -> None:
    ws, rank, _ = _dist()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    res = cpu_oracle_rate(ENVS_PER_GPU, args.warmup, args.steps, threads)
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "envs_per_gpu": ENVS_PER_GPU, "frameskip": FRAMES},
        "cpu_baseline": res,
        "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference Warp runtime is not installable offline; this arm is the C restatement of the "
                "reference step (oracle/) on all host threads",
    }
    print(json.dumps(line), flush=True)


def run_gbx(args) -> None:
    import torch

    from gbxcule_b200 import GbxVecCudaBackend, roms
    from gbxcule_b200.multi import job_rate, rank_seed, reduce_run_stats

    ws, rank, local = _dist()
    dist = None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n = ENVS_PER_GPU
    K, W = args.steps, args.warmup
    rom = roms.CONFIG_ROMS[CONFIG]()
    rng = np.random.default_rng(rank_seed(0, rank))  # this rank's own env slice
    acts_host = np.stack([roms.uniform_actions(rng, n, 9) for _ in range(W + 2 * K)])
    be = GbxVecCudaBackend(rom, num_envs=n, frames_per_step=FRAMES, release_after_frames=RELEASE,
                           render_pixels_packed=True, render_on_step=False, device=f"cuda:{local}")
    be.reset()
    acts_dev = torch.as_tensor(acts_host, device=dev)
    for w in range(W):
        be.step_torch(acts_dev[w])
        be.render_pixels_snapshot_torch()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    i64 = be._view("i64")  # row 0: per-env emulated instruction counters
    ninstr0 = int(i64[0].sum())
    clocks = ClockSampler(local)
    clocks.start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    wall0 = time.perf_counter()
    for k in range(K):
        flush.zero_()  # L2 flush between timed steps, outside the events
        s, m, e = ev[k]
        s.record()
        be.step_torch(acts_dev[W + k])
        m.record()
        be.render_pixels_snapshot_torch()
        e.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    clk = clocks.stop()
    step_ms = [s.elapsed_time(m) for s, m, _ in ev]
    total_ms = sum(s.elapsed_time(e) for s, _, e in ev)
    ninstr = int(i64[0].sum()) - ninstr0

    # end to end through the public API with host buffers
    acts_pin = torch.from_numpy(acts_host[W + K:W + 2 * K]).pin_memory()
    out_dev = torch.empty((n, 72, 20), dtype=torch.uint8, device=dev)
    out_host = torch.empty((2, n, 72, 20), dtype=torch.uint8).pin_memory()
    a_dev = torch.empty((n,), dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for k in range(K):
        a_dev.copy_(acts_pin[k], non_blocking=True)
        be.step_torch(a_dev)
        be.render_pixels_snapshot_packed_to_torch(out_dev)
        out_host[k % 2].copy_(out_dev, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    (total_ms, e2e_ms, step_avg_ms), (ninstr,) = reduce_run_stats(
        dist, dev, [total_ms, e2e_ms, float(np.mean(step_ms))], [ninstr])
    be.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    total_envs = n * ws
    value = job_rate(n, ws, K, total_ms)
    peaks = _peaks()
    achieved = STEP_STATE_BYTES * n / (step_avg_ms / 1e3) / 1e9
    traffic = STEP_KERNEL_DRAM_BYTES_4096 * n / 4096
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": K, "warmup": W,
        "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "envs_per_gpu": n, "frameskip": FRAMES, "release_after_frames": RELEASE,
                   "obs": "packed 2bpp 72x20 rendered every step", "l2": "flushed between timed steps (256 MiB write)",
                   "parallelism": f"{ws} independent env slices, no collective on the step path"},
        "emulated_frames_per_s": value * FRAMES,
        # SM83 instructions retired by all envs per second of step-kernel time
        # (the step kernel is bound by integer issue per emulated instruction)
        "emulated_instr_per_s": ninstr / (step_avg_ms * K / 1e3),
        "emulated_instr_per_env_step": ninstr / (total_envs * K),
        "e2e": {"value": job_rate(n, ws, K, e2e_ms), "unit": UNIT, "h2d_bytes_per_step": 4 * n,
                "d2h_bytes_per_step": 72 * 20 * n},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                     "peak_source": peaks["source"], "kernel": "gb_step_kernel",
                     "kernel_ms": step_avg_ms, "bytes_per_env_step": STEP_STATE_BYTES},
        # the binding roof: warp-instruction issue slots used by the step
        # kernel (emulated instructions/s x warp instructions per emulated
        # instruction) over the SMs' issue slots at the sampled SM clock
        "issue_roofline": _issue_roofline(ninstr / (step_avg_ms * K / 1e3) / ws, clk),
        "clocks": clk,
        "gpu_launches": 2 * K,
        "wall_s_timed": wall,
    }
    if ws == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_oracle_rate(n, 3, 2, os.cpu_count() or 1)
    print(json.dumps(line), flush=True)


def run_rollout_workload(args) -> None:
    """Benchmark config 5: policy rollouts on the MBC3 + PPU cartridge.

    Per env-step: packed render -> 2 bpp unpack -> bf16 conv policy -> sampled
    actions -> step_torch -> masked restore of a seeded 5 % of envs from a
    snapshot taken after warm-up. Timed end to end with CUDA events; the
    policy and the restores are inside the timed region.
    """
    import torch

    from gbxcule_b200 import GbxVecCudaBackend, ResetCache, roms
    from gbxcule_b200.multi import job_rate, rank_seed, reduce_run_stats
    from gbxcule_b200.rollout import make_policy, run_rollout

    ws, rank, local = _dist()
    dist = None
    torch.cuda.set_device(local)
    if ws > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.backends.cudnn.benchmark = True  # the policy's conv shapes repeat every step
    n = args.envs or 131072
    K, W = args.steps, args.warmup
    be = GbxVecCudaBackend(roms.config5_rom(), num_envs=n, frames_per_step=FRAMES,
                           release_after_frames=RELEASE, render_on_step=False, device=f"cuda:{local}")
    be.reset()
    pol = make_policy(dev, seed=rank_seed(5, rank))
    gen = torch.Generator(device=dev).manual_seed(rank_seed(1005, rank))
    packed = torch.empty((n, 72, 20), dtype=torch.uint8, device=dev)
    run_rollout(be, pol, W, generator=gen, packed_out=packed)
    cache = ResetCache.from_backend(be, env_idx=0)
    masks = [torch.as_tensor(np.random.default_rng(rank_seed(2005, rank) + k).random(n) < 0.05, device=dev)
             for k in range(K)]
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run_rollout(be, pol, K, generator=gen, reset_cache=cache, reset_mask=lambda k: masks[k], packed_out=packed)
    e1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    (ms,), _ = reduce_run_stats(dist, dev, [e0.elapsed_time(e1)], [])
    cache.close()
    be.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    value = job_rate(n, ws, K, ms)
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u8", "data": "synthetic",
        "config": {"workload": f"config5: MBC3 + PPU cartridge, {n} envs/GPU, frameskip 24, bf16 conv policy "
                               "on packed frames, sampled actions, 5 % masked restores per step",
                   "envs_per_gpu": n, "policy": "Conv(1-32,k4,s2)-Conv(32-64,k3,s2)-Conv(64-64,k3,s1)-"
                   "Linear(512)-Linear(9), bf16, random init"},
        "emulated_frames_per_s": value * FRAMES, "clocks": clk}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="gbx", choices=["gbx", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="config2", choices=["config2", "config5"],
                    help="config2 (default): the benchmark line; config5: policy rollouts")
    ap.add_argument("--envs", type=int, default=0, help="envs per GPU for --workload config5")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "config5":
        run_rollout_workload(args)
    else:
        run_gbx(args)


if __name__ == "__main__":
    main()
