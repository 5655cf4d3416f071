"""Multi-GPU host logic: one process per GPU, environments sharded by rank.

Environments are independent, so a job of ``world_size`` ranks gives each rank
its own contiguous slice of ``envs_per_rank`` envs on its own GPU (its own
``GbxVecCudaBackend``; no peer memory, no collective on the step path). The
only cross-rank traffic is what a benchmark or a stats pass needs at the end:
the slowest rank's times (max) and the job's counters (sum).

``dist`` arguments are ``torch.distributed`` (or ``None`` for one process);
the same code runs under NCCL on GPUs and under gloo in the CPU tests.
"""

from __future__ import annotations

from typing import Sequence


def rank_env_slice(rank: int, world_size: int, envs_per_rank: int) -> tuple[int, int]:
    """Global env range [lo, hi) owned by ``rank`` (weak scaling: fixed per rank)."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} out of range for world size {world_size}")
    if envs_per_rank <= 0:
        raise ValueError(f"envs_per_rank must be > 0, got {envs_per_rank}")
    lo = rank * envs_per_rank
    return lo, lo + envs_per_rank


def rank_seed(base_seed: int, rank: int) -> int:
    """Seed of a rank's action stream: distinct per rank, reproducible per job."""
    return int(base_seed) + int(rank)


def reduce_run_stats(dist, device, max_values: Sequence[float], sum_values: Sequence[float]
                     ) -> tuple[list[float], list[float]]:
    """Max over ranks of ``max_values`` (times) and sum of ``sum_values`` (counters).

    Every rank must call this with the same number of values, in the same
    order. With ``dist`` None the inputs come back unchanged.
    """
    mx = [float(v) for v in max_values]
    sm = [float(v) for v in sum_values]
    if dist is None:
        return mx, sm
    import torch

    t = torch.tensor(mx, dtype=torch.float64, device=device)
    c = torch.tensor(sm, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(c, op=dist.ReduceOp.SUM)
    return [float(x) for x in t.tolist()], [float(x) for x in c.tolist()]


def job_rate(envs_per_rank: int, world_size: int, steps: int, max_ms: float) -> float:
    """Whole-job env-steps/s: every rank's envs over the slowest rank's time."""
    if max_ms <= 0:
        raise ValueError(f"time must be > 0 ms, got {max_ms}")
    return envs_per_rank * world_size * steps / (max_ms / 1e3)
