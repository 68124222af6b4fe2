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


def _gather_equal(local: torch.Tensor) -> torch.Tensor:
    """All ranks' equally shaped blocks concatenated along dim 0: one collective,
    no host synchronisation."""
    world = dist.get_world_size()
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous())
    return out


def gather_outputs(local: torch.Tensor, sizes=None) -> torch.Tensor:
    """Concatenate every rank's per-sequence outputs along dim 0, in rank order.
    Ranks may own different numbers of sequences; `sizes` (every rank's count,
    e.g. from shard_range) saves the exchange of the counts, and equal counts
    take a single collective."""
    if not _ready():
        return local
    world = dist.get_world_size()
    if sizes is not None and len(set(sizes)) == 1:
        return _gather_equal(local)
    if sizes is None:
        n = torch.tensor([local.shape[0]], dtype=torch.int64, device=local.device)
        got = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(got, n)
        sizes = [int(x.item()) for x in got]
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
    if len(set(counts)) == 1:   # equal blocks: one collective into [world, B, c, D], then heads in rank order
        out = _gather_equal(local).view((world,) + tuple(local.shape))
        return out.permute(1, 0, 2, 3).reshape(local.shape[0], world * local.shape[1], *local.shape[2:])
    mx = max(counts)
    pad = torch.zeros((local.shape[0], mx) + tuple(local.shape[2:]), dtype=local.dtype, device=local.device)
    pad[:, :local.shape[1]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad.contiguous())
    return torch.cat([p[:, :c] for p, c in zip(parts, counts)], dim=1)
