"""Row sharding across GPUs of one node: the host logic of the N-GPU path.

Rows of these ops are independent, so N GPUs split a token batch into N
contiguous row blocks and run the same kernel on each, with no collective on
the data path (weights and RoPE tables are replicated per GPU). The only
cross-rank communication is on the host side of a measurement: a barrier
and the max of the per-rank device times. One process per GPU, launched by
``torch.distributed.run``; the same functions run over ``gloo`` on CPU.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def shard_range(total_rows: int, world: int, rank: int) -> tuple[int, int]:
    """``[start, stop)`` of rank ``rank``'s contiguous block; blocks differ by at most one row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    base, extra = divmod(total_rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def env_world() -> tuple[int, int, int]:
    """``(world_size, rank, local_rank)`` from the launcher's environment (1, 0, 0 without one)."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str, *, timeout_s: float = 180.0, device: torch.device | None = None) -> tuple[int, int, int]:
    """Join the process group when the launcher started more than one rank."""
    world, rank, local = env_world()
    if world > 1 and not dist.is_initialized():
        kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if device is not None and device.type == "cuda":
            kwargs["device_id"] = device
        dist.init_process_group(backend, **kwargs)
    return world, rank, local


def barrier() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.barrier()


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    """Largest ``value`` over all ranks (the job's time is its slowest rank's)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device: torch.device | None = None) -> float:
    """Sum of ``value`` over all ranks (the bytes of a step over all shards)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item()) if not isinstance(value, int) else int(round(t.item()))


def all_over_ranks(flag: bool, device: torch.device | None = None) -> bool:
    """True when ``flag`` holds on every rank (a per-shard check)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return bool(flag)
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def finish() -> None:
    if dist.is_available() and dist.is_initialized():
        dist.destroy_process_group()
