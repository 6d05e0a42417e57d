"""Multi-GPU sharding of the decode step by (batch, kv-head) units.

Decode attention has no cross-unit dependency: a unit is one sequence's KV
head together with the query heads that read it. Ranks therefore own disjoint,
contiguous unit ranges and never exchange data on the hot path. This module
holds the host-side pieces used by bench.py and usable by a serving loop:

* ``unit_range`` / ``batch_range``: which units (or whole sequences) a rank owns;
* ``slab_seed``: a per-(batch, kv-head) seed, so any rank (or a CPU checker)
  can regenerate any slab independently of the number of ranks;
* ``gather_shards``: all-gather of per-rank output shards (verification only,
  off the hot path);
* ``max_over_ranks``: the job time of a step is the slowest rank's.

Everything works with any torch.distributed backend (NCCL on GPUs, gloo for
the CPU tests).
"""
from __future__ import annotations

from typing import Optional, Tuple


def unit_range(n_units: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, balanced [start, end) of ``n_units`` for ``rank``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    return rank * n_units // world, (rank + 1) * n_units // world


def batch_range(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Sequences owned by ``rank`` when whole sequences are sharded (every KV
    head of a sequence on the same rank, so q/out shards are contiguous)."""
    if batch % world:
        raise ValueError(f"batch {batch} is not divisible by world size {world}")
    per = batch // world
    return rank * per, (rank + 1) * per


def slab_seed(base_seed: int, batch_index: int, kv_head: int, n_kv_heads: int) -> int:
    """Seed of the (batch, kv-head) slab: base + global slab index."""
    return base_seed + batch_index * n_kv_heads + kv_head


def max_over_ranks(value: float, device=None, group=None) -> float:
    """MAX all-reduce of a scalar (a per-rank time)."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_shards(shard, group=None):
    """All-gather equally shaped per-rank shards along dim 0 (rank order)."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized():
        return shard
    world = dist.get_world_size(group)
    shape = torch.tensor(list(shard.shape), dtype=torch.int64, device=shard.device)
    shapes = [torch.empty_like(shape) for _ in range(world)]
    dist.all_gather(shapes, shape, group=group)
    for r, sh in enumerate(shapes):
        if not torch.equal(sh, shape):
            raise RuntimeError(f"rank {r} shard shape {sh.tolist()} differs from {shape.tolist()}")
    parts = [torch.empty_like(shard) for _ in range(world)]
    dist.all_gather(parts, shard.contiguous(), group=group)
    return torch.cat(parts, dim=0)


def init_from_env(backend: str, timeout_s: Optional[float] = None):
    """Initialise the default process group from torchrun's environment
    (RANK, WORLD_SIZE, MASTER_ADDR/PORT). Returns (world, rank)."""
    import datetime
    import os

    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kw = {}
        if timeout_s is not None:
            kw["timeout"] = datetime.timedelta(seconds=timeout_s)
        dist.init_process_group(backend, **kw)
    return world, rank
