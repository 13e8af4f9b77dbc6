"""Request sharding across GPUs: one process per GPU, rows independent.

The decoding step has no exchange between rows, so a multi-GPU deployment is N
independent batches: every rank owns a contiguous block of the global request
rows and its own replicated grammar tables. ``torch.distributed`` is used only
off the hot path -- barriers around a measured region and reductions of
per-rank timings / counters.
"""

from __future__ import annotations

import datetime
import os

import torch


def dist_info() -> tuple[int, int, int]:
    """(rank, world size, local rank) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str, device: torch.device | None = None, timeout_s: float = 120.0) -> bool:
    """Join the process group when running under torchrun (world size > 1);
    returns whether a group exists. The short timeout turns a rank that never
    arrives into an error on the others instead of a hang."""
    import torch.distributed as dist

    _, world, _ = dist_info()
    if world <= 1:
        return False
    if not dist.is_initialized():
        kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if device is not None and backend == "nccl":
            kw["device_id"] = device
        dist.init_process_group(backend, **kw)
    return True


def shard_rows(total_rows: int, world: int, rank: int) -> range:
    """The contiguous block of global rows rank `rank` owns (sizes differ by
    at most one)."""
    base, extra = divmod(total_rows, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def _reduce(values: list[float], op: str, device: torch.device | None) -> list[float]:
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(values)
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return [float(x) for x in t.tolist()]


def max_over_ranks(values: list[float], device: torch.device | None = None) -> list[float]:
    """Element-wise maximum over ranks (identity without a process group)."""
    return _reduce(values, "max", device)


def sum_over_ranks(values: list[float], device: torch.device | None = None) -> list[float]:
    """Element-wise sum over ranks (identity without a process group)."""
    return _reduce(values, "sum", device)


def gather_over_ranks(value: float, device: torch.device | None = None) -> list[float]:
    """``value`` of every rank, in rank order (``[value]`` without a group)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [float(value)]
    t = torch.zeros(dist.get_world_size(), dtype=torch.float64, device=device)
    t[dist.get_rank()] = value
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return [float(x) for x in t.tolist()]


def barrier() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def finish() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
