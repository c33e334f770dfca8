"""CPU: the multi-GPU host logic (contiguous shards, max over ranks) on a
world-size-2 gloo process group over 127.0.0.1."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fast_moss_b200.shards import max_over_ranks, shard, shard_bounds


def test_shard_bounds_cover_every_item_once():
    for total in (0, 1, 7, 64, 8192, 10001):
        for world in (1, 2, 3, 4, 8):
            seen = []
            sizes = []
            for rank in range(world):
                start, end = shard_bounds(total, rank, world)
                seen.extend(range(start, end))
                sizes.append(end - start)
            assert seen == list(range(total))
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def test_max_over_ranks_without_a_group_is_identity():
    assert max_over_ranks([1.5, 2]) == [1.5, 2.0]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        clips = torch.arange(64 * 3).reshape(64, 3)  # 64 independent clips
        mine = shard(clips, rank, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine[:, 0].tolist())
        t = max_over_ranks([0.1 * (rank + 1), 5.0 - rank])
        if rank == 0:
            out.put((sum(gathered, []), t))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    items, t = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert items == [3 * i for i in range(64)]  # every clip once, in order
    assert t == pytest.approx([0.2, 5.0])
