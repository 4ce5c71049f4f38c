"""Host-side multi-rank helpers: batch sharding, max-over-ranks timing, gathers.

The hot path partitions by sequence: every (b, h) sequence is independent in all
four ops, so ranks split the batch and run with no collective on the data path.
Collectives here are only for timing (max over ranks) and for checking results
(gather to rank 0), outside any timed region. Works with any torch.distributed
backend (nccl on GPUs, gloo on CPUs for tests).
"""
from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def world() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment (1 process: 0, 1, 0)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str, timeout_s: float = 120.0, device=None) -> None:
    """init_process_group with a short timeout, so a rank that dies or never joins
    turns the next collective into an error instead of a hang."""
    kw = dict(backend=backend, timeout=timedelta(seconds=timeout_s))
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    dist.init_process_group(**kw)


def shard_range(n: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) share of n units for `rank`; sizes differ by at most one."""
    assert world_size >= 1 and 0 <= rank < world_size and n >= 0
    base, extra = divmod(n, world_size)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def max_over_ranks(x: float, device=None) -> float:
    """Max of a scalar over all ranks (the bench's elapsed time)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_batches(t: torch.Tensor, device=None):
    """Concatenate every rank's batch shard (dim 0) on rank 0; None on other ranks.
    Shards may differ in size by one (shard_range)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return t
    ws, rank = dist.get_world_size(), dist.get_rank()
    n = torch.tensor([t.shape[0]], dtype=torch.int64, device=device)
    sizes = [torch.zeros_like(n) for _ in range(ws)]
    dist.all_gather(sizes, n)
    mx = int(max(s.item() for s in sizes))
    pad = torch.zeros((mx,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    pad[: t.shape[0]] = t
    bufs = [torch.empty_like(pad) for _ in range(ws)]
    dist.all_gather(bufs, pad)
    if rank != 0:
        return None
    return torch.cat([b[: int(s.item())] for b, s in zip(bufs, sizes)], 0)
