"""Sequence sharding across GPUs (one process per GPU).

Every (sequence, layer, KV head) unit of the compressed KV path is independent
(compressed_attention.py:21-22 keeps no cross-head state), so a batch is split
by sequence: rank r owns a contiguous block of sequences, holds their tiers in
its own HBM and decodes them with no data-path collective.  The only
collectives are for reporting: the max over ranks of a device time and an
all-gather of per-step outputs.  They run over NCCL between GPUs and over gloo
on CPU (tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n_items: int, world: int, rank: int) -> range:
    """Contiguous block of items [start, stop) owned by `rank`; blocks differ in
    size by at most one and cover 0..n_items-1 exactly once."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_items < 0:
        raise ValueError(f"n_items={n_items}")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def _ready() -> bool:
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


def max_over_ranks(value: float, device=None) -> float:
    """The largest `value` of all ranks (the job's time is its slowest rank's)."""
    if not _ready():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_outputs(local: torch.Tensor) -> torch.Tensor:
    """Concatenate every rank's per-sequence outputs along dim 0, in rank order
    (ranks may own different numbers of sequences)."""
    if not _ready():
        return local
    world = dist.get_world_size()
    n = torch.tensor([local.shape[0]], dtype=torch.int64, device=local.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n)
    sizes = [int(s.item()) for s in sizes]
    mx = max(sizes)
    pad = torch.zeros((mx,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[:local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], dim=0)
