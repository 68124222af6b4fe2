"""Sequence and KV-head sharding host logic on CPU: world-size-2 gloo ranks (no GPU)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helix_online_kv.sharding import gather_heads, gather_outputs, head_shard, max_over_ranks, shard_range


def test_shard_range_partitions():
    for n in (0, 1, 7, 8, 64, 65):
        for world in (1, 2, 3, 8):
            got = [i for r in range(world) for i in shard_range(n, world, r)]
            assert got == list(range(n)), (n, world)
            sizes = [len(shard_range(n, world, r)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_seq, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        mine = shard_range(n_seq, world, rank)
        # per-sequence "outputs": the sequence index in every element
        out = torch.tensor([[float(i)] * 3 for i in mine]).reshape(len(mine), 3)
        full = gather_outputs(out)
        sizes = [len(shard_range(n_seq, world, r)) for r in range(world)]
        assert gather_outputs(out, sizes=sizes).tolist() == full.tolist()
        t = max_over_ranks(1.5 + rank)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, full.tolist(), t, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, None, repr(e)))


@pytest.mark.parametrize("n_seq", [8, 5])
def test_two_gloo_ranks(n_seq):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, n_seq, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, full, t, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert full == [[float(i)] * 3 for i in range(n_seq)]
        assert t == 2.5


def _head_worker(rank, world, port, n_kv, G, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        mine = head_shard(n_kv, world, rank)
        # this rank's query heads of 2 sequences: every element = its global query head
        hq = [h * G + g for h in mine for g in range(G)]
        local = torch.tensor([[[float(x)] * 3 for x in hq]] * 2).reshape(2, len(hq), 3)
        full = gather_heads(local, n_kv, G)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, full.tolist(), None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


@pytest.mark.parametrize("n_kv,G", [(8, 4), (3, 8), (1, 4)])
def test_head_partition_two_gloo_ranks(n_kv, G):
    """KV-head partition (fewer sequences than GPUs): the heads are covered
    once, and the per-layer all-gather reassembles [B, H_q, D] in head order,
    also when a rank owns no head."""
    got = [i for r in range(2) for i in head_shard(n_kv, 2, r)]
    assert got == list(range(n_kv))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_head_worker, args=(r, 2, port, n_kv, G, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    want = [[[float(x)] * 3 for x in range(n_kv * G)]] * 2
    for rank, full, err in res:
        assert err is None, f"rank {rank}: {err}"
        assert full == want
