"""Views data-parallel training across the GPUs of one box.

Every rank holds the whole pool (the Gaussians are replicated); each step every
rank renders its own camera view and writes its gradient rows, the rows are
summed over ranks with one all-reduce (NCCL over NVLink), and every rank runs
the same fused Adam on the summed rows scaled by 1/world, so the replicas stay
bit-identical without any parameter broadcast.  The densification statistics
(grad2d, count) are summed before each densify step, and the densify noise is
drawn from a generator seeded by the step, identically on every rank.

The functions here hold that host-side logic; they work with any
``torch.distributed`` backend (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.distributed as dist


def world_of(pg) -> int:
    return 1 if pg is None else dist.get_world_size(pg)


def rank_of(pg) -> int:
    return 0 if pg is None else dist.get_rank(pg)


def view_for(step: int, rank: int, world: int, num_views: int) -> int:
    """The camera view rank ``rank`` trains on at ``step``: the world's ranks
    take consecutive views, and consecutive steps advance by ``world``."""
    return (rank + world * step) % num_views


def reduce_gradient_rows(grad_rows: torch.Tensor, pg) -> float:
    """Sums the gradient rows of all ranks in place; returns the scale Adam
    applies to them (1/world, so the update follows the mean over views)."""
    w = world_of(pg)
    if w > 1:
        dist.all_reduce(grad_rows, op=dist.ReduceOp.SUM, group=pg)
    return 1.0 / w


def reduce_densify_stats(grad2d: torch.Tensor, count: torch.Tensor, pg) -> None:
    """Sums the per-slot densification statistics over ranks in place."""
    if world_of(pg) > 1:
        dist.all_reduce(grad2d, op=dist.ReduceOp.SUM, group=pg)
        dist.all_reduce(count, op=dist.ReduceOp.SUM, group=pg)


def densify_noise(step: int, n: int, device) -> Dict[str, torch.Tensor]:
    """The normal draws of one densify step (child means x2, child quaternion),
    from a generator seeded by the step so every rank draws the same values."""
    gen = torch.Generator(device=device)
    gen.manual_seed(1_000_003 * int(step) + 17)
    return {"means1": torch.randn((n, 3), generator=gen, device=device),
            "means2": torch.randn((n, 3), generator=gen, device=device),
            "quats2": torch.randn((n, 4), generator=gen, device=device)}


def init_from_env(backend: str = "nccl", timeout_s: float = 180.0):
    """Initialise the default process group from torchrun's environment
    (RANK, WORLD_SIZE, LOCAL_RANK, MASTER_ADDR/PORT); returns (rank, world,
    local_rank, group or None for a single process)."""
    import datetime
    import os
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1:
        return rank, world, local, None
    kw = {}
    if backend == "nccl":
        torch.cuda.set_device(local)
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank, world, local, dist.group.WORLD


def max_over_ranks(x: float, pg, device: Optional[torch.device] = None) -> float:
    if world_of(pg) == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=pg)
    return float(t.item())
