"""Env sharding across GPUs (one process per GPU): rank r owns envs [r*n, (r+1)*n) through env_offset, whose RNG
streams are default_rng(seed*1000 + r*n + i) - exactly the streams of one big run (the reference's env_offset
contract, env.py:155-156, tests/test_api.py:89-98). There is no collective on the env path; the only
cross-rank operation is the timing reduction (max over ranks) used by the benchmark."""
from __future__ import annotations


def env_offset(rank: int, n_per_rank: int) -> int:
    return rank * n_per_rank


def shard_seeds(seed: int, rank: int, n_per_rank: int) -> list[int]:
    off = env_offset(rank, n_per_rank)
    return [seed * 1000 + off + i for i in range(n_per_rank)]


def max_over_ranks(value: float, device=None) -> float:
    """All-reduce MAX of a per-rank float (elapsed ms); identity without an initialised process group."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(world: int, n_per_rank: int, steps: int, max_ms: float) -> float:
    """Whole-job env-steps/s: all envs of all ranks over the slowest rank's time (weak scaling)."""
    return world * n_per_rank * steps / (max_ms / 1000.0)
