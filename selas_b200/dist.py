"""Multi-GPU plumbing for the image-sharded FLUX step: one process per GPU, images split across ranks,
no collective on the data path (the path is partitioned: every image's denoise is independent).

Only three host-side pieces are shared: which images a rank owns, the max-over-ranks reduction of a
timing (the job takes as long as its slowest rank) and the per-rank values behind it (which rank, at
which clock, set the pace).
"""

from __future__ import annotations

import torch


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


def per_rank(value: float | None, device: torch.device | str = "cpu") -> list[float | None]:
    """`value` from every rank, in rank order (a one-element list without a process group). None (a
    rank that has no figure, e.g. no clock samples) travels as NaN and comes back as None."""
    import torch.distributed as td

    v = float("nan") if value is None else float(value)
    if not (td.is_available() and td.is_initialized()) or td.get_world_size() == 1:
        return [None if value is None else v]
    mine = torch.tensor([v], dtype=torch.float64, device=device)
    every = [torch.empty_like(mine) for _ in range(td.get_world_size())]
    td.all_gather(every, mine)
    out = [float(t.item()) for t in every]
    return [None if x != x else x for x in out]
