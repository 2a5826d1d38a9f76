"""Replica serving across GPUs (config 4): independent engines, no collectives on the data path.

At bs=1 the path does not shard (one observation, a sequential 10-step loop, an
18-layer dependency chain), so N GPUs serve N independent streams of
observations.  A batch of B observations is split contiguously over the ranks;
each rank runs its share through its own engine.  ``torch.distributed`` is used
only for the start barrier and the max-over-ranks timing.
"""

from __future__ import annotations

from typing import Callable, List, Optional


def shard_range(n_items: int, world: int, rank: int) -> range:
    """Contiguous block of item indices owned by ``rank`` (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, rem = divmod(n_items, world)
    start = rank * base + min(rank, rem)
    return range(start, start + base + (1 if rank < rem else 0))


def max_over_ranks(value: float, pg=None, device=None) -> float:
    """Max of a per-rank scalar (the job's time is its slowest rank's)."""
    if pg is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64, device=device)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def gather_outputs(local: List, pg=None) -> List:
    """Host-side gather of per-rank results (list of CPU tensors) to every rank, rank order."""
    if pg is None:
        return list(local)
    out: List[Optional[List]] = [None] * pg.get_world_size()
    pg.all_gather_object(out, list(local))
    return [x for part in out for x in part]


def serve(n_obs: int, run_one: Callable[[int], object], pg=None) -> List:
    """Run observations ``shard_range(n_obs)`` of this rank through ``run_one`` and gather all."""
    rank = pg.get_rank() if pg is not None else 0
    world = pg.get_world_size() if pg is not None else 1
    local = [run_one(i) for i in shard_range(n_obs, world, rank)]
    return gather_outputs(local, pg)
