"""Multi-rank host logic on CPU: two gloo ranks run the same slicing and
reduction code the NCCL benchmark runs on GPUs (gbxcule_b200.multi)."""

from __future__ import annotations

import multiprocessing as mp
import os
import socket

import pytest

from gbxcule_b200 import multi


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        lo, hi = multi.rank_env_slice(rank, world, 4096)
        # rank r "took" 100 + 10 r ms and retired 1000 + r instructions
        (t_max, e_max), (instr,) = multi.reduce_run_stats(
            dist, torch.device("cpu"), [100.0 + 10 * rank, 50.0 - rank], [1000.0 + rank])
        out.put((rank, lo, hi, t_max, e_max, instr, multi.rank_seed(7, rank)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_slice_and_reduce():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(out.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    slices = [(lo, hi) for _, lo, hi, *_ in res]
    assert slices == [(0, 4096), (4096, 8192)]  # disjoint, contiguous, fixed per rank
    for _, _, _, t_max, e_max, instr, _ in res:
        assert t_max == 110.0 and e_max == 50.0  # slowest rank's time on every rank
        assert instr == 2001.0                   # job total
    assert [seed for *_, seed in res] == [7, 8]


def test_single_process_identity_and_job_rate():
    mx, sm = multi.reduce_run_stats(None, None, [3.0, 4.0], [5.0])
    assert mx == [3.0, 4.0] and sm == [5.0]
    # 2 ranks x 4,096 envs x 10 steps over the slowest rank's 1,000 ms
    assert multi.job_rate(4096, 2, 10, 1000.0) == 81920.0
    with pytest.raises(ValueError):
        multi.rank_env_slice(2, 2, 16)
    with pytest.raises(ValueError):
        multi.job_rate(1, 1, 1, 0.0)


# ---------------------------------------------------------------------------
# Sharded emulation equals one process: two gloo ranks each step their own
# contiguous env slice on the oracle with their own action stream
# (rank_seed), and the gathered states equal one process stepping all the
# global env ids with the same per-slice streams.
# ---------------------------------------------------------------------------
ENVS_PER_RANK, STEPS, CFG = 3, 3, 4


def _slice_actions(rank: int) -> list:
    import numpy as np

    from gbxcule_b200 import roms

    rng = np.random.default_rng(multi.rank_seed(11, rank))
    return [roms.uniform_actions(rng, ENVS_PER_RANK, 9) for _ in range(STEPS)]


def _per_env_fields(s: dict, n: int) -> dict:
    """Per-env arrays of a canonical state, [n, ...] each (env-0 latches are per batch)."""
    import numpy as np

    from gbxcule_b200 import state as st

    return {k: np.asarray(s[k]).reshape(n, -1) for k in st.ORDER if not k.startswith("latch_")}


def _shard_main(rank: int, world: int, port: int, out) -> None:
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from gbxcule_b200 import roms
    from oracle import OracleEnvs

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        lo, hi = multi.rank_env_slice(rank, world, ENVS_PER_RANK)
        o = OracleEnvs(roms.CONFIG_ROMS[CFG](), roms.boot_stub(), hi - lo, threads=1)
        for a in _slice_actions(rank):
            o.step(a, 24, 8)
        mine = _per_env_fields(o.state(), hi - lo)
        parts = [None] * world
        dist.all_gather_object(parts, (lo, hi, mine))
        if rank == 0:
            out.put(parts)
    finally:
        dist.destroy_process_group()


def test_sharded_slices_equal_one_process():
    import numpy as np

    from gbxcule_b200 import roms
    from oracle import OracleEnvs

    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_shard_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    parts = out.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # one process, all global env ids, each slice driven by its rank's stream
    n = world * ENVS_PER_RANK
    o = OracleEnvs(roms.CONFIG_ROMS[CFG](), roms.boot_stub(), n, threads=2)
    streams = [_slice_actions(r) for r in range(world)]
    for k in range(STEPS):
        o.step(np.concatenate([streams[r][k] for r in range(world)]), 24, 8)
    whole = _per_env_fields(o.state(), n)
    for lo, hi, mine in parts:
        for name, arr in mine.items():
            assert np.array_equal(arr, whole[name][lo:hi]), f"slice [{lo}, {hi}) field {name}"
