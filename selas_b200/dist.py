"""Multi-GPU plumbing for the image-sharded FLUX step: one process per GPU, images split across ranks,
no collective on the data path (the path is partitioned: every image's denoise is independent).

Only three host-side pieces are shared: which images a rank owns, the barrier that brackets a timed
region, and the max-over-ranks reduction of a timing (the job takes as long as its slowest rank).
"""

from __future__ import annotations

import os

import torch


def world() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment (1-process defaults)."""
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def shard(n_images: int, rank: int, world_size: int) -> range:
    """Contiguous block of image indices owned by `rank`; the first `n % world` ranks get one extra."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} of {world_size}")
    base, extra = divmod(n_images, world_size)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """The maximum of `value` over all ranks (identity without an initialised process group)."""
    import torch.distributed as td

    if not (td.is_available() and td.is_initialized()) or td.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    td.all_reduce(t, op=td.ReduceOp.MAX)
    return float(t.item())


def gather_sum(value: float, device: torch.device | str = "cpu") -> float:
    """The sum of `value` over all ranks (identity without a process group)."""
    import torch.distributed as td

    if not (td.is_available() and td.is_initialized()) or td.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    td.all_reduce(t, op=td.ReduceOp.SUM)
    return float(t.item())
