"""Multi-GPU plumbing: one process per GPU, batch-sharded.

Every row of a Mamba block's (or a residual stack's) batch is independent,
so N GPUs split the batch into N contiguous shards and run with no
collective on the data path.  The only collectives are bookkeeping: a barrier
around timed regions and the max of the ranks' device times.  Works with the
``nccl`` backend on GPUs and ``gloo`` on CPU (the host logic is tested that
way).
"""
from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def env() -> tuple:
    """(world_size, rank, local_rank) from the launcher's environment
    (torchrun sets WORLD_SIZE / RANK / LOCAL_RANK; defaults: one process)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str = "nccl", device: torch.device | None = None,
         timeout_s: float = 120.0) -> None:
    """Join the process group (no-op for a single process).  A short timeout
    makes ranks that wait on a missing peer fail instead of hanging."""
    ws, _, _ = env()
    if ws > 1 and not dist.is_initialized():
        kw = {"device_id": device} if backend == "nccl" and device is not None else {}
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s), **kw)


def shutdown() -> None:
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def shard(total: int, world: int, rank: int) -> tuple:
    """[start, stop) of rank's contiguous share of ``total`` batch rows; the
    first ``total % world`` ranks take one row more.  Shards are disjoint and
    cover 0..total."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} not in a world of {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    """The largest ``value`` of all ranks (the job's time is its slowest
    rank's); the value itself for a single process."""
    if not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device: torch.device | None = None) -> float:
    if not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
