"""Sequence and KV-head sharding across GPUs (one process per GPU).

Every (sequence, layer, KV head) unit of the compressed KV path is independent
(compressed_attention.py:21-22 keeps no cross-head state).  A batch is split
by sequence (the primary partition): rank r owns a contiguous block of
sequences, holds their tiers in its own HBM and decodes them with no
data-path collective; per-step outputs are all-gathered for reporting.  With
fewer sequences than GPUs the KV heads are split instead (the secondary
partition): rank r owns a contiguous block of KV heads and their query heads,
and every layer's attention outputs [B, H_q, D] are all-gathered along the
head axis.  The collectives run over NCCL between GPUs and over gloo on CPU
(tests).
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


def head_shard(n_kv_heads: int, world: int, rank: int) -> range:
    """KV heads [start, stop) owned by `rank` in the head partition (the same
    contiguous split as shard_range)."""
    return shard_range(n_kv_heads, world, rank)


def gather_heads(local: torch.Tensor, n_kv_heads: int, q_per_kv: int) -> torch.Tensor:
    """Reassemble [B, H_q, D] attention outputs from every rank's [B, G * h_r, D]
    block (h_r = the rank's KV heads, G = q_per_kv query heads per KV head), in
    head order.  A rank may own no head (fewer KV heads than ranks)."""
    if not _ready():
        return local
    world = dist.get_world_size()
    counts = [len(head_shard(n_kv_heads, world, r)) * q_per_kv for r in range(world)]
    mx = max(counts)
    pad = torch.zeros((local.shape[0], mx) + tuple(local.shape[2:]), dtype=local.dtype, device=local.device)
    pad[:, :local.shape[1]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad.contiguous())
    return torch.cat([p[:, :c] for p, c in zip(parts, counts)], dim=1)
