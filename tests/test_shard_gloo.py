"""Multi-rank host logic of the batch-sharded path, on CPU with the gloo
backend (world size 2 and 3): shard bounds cover the batch exactly once, and
values gathered from ragged shards come back complete and in rank order."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from d2p_b200.shard import gather_values, shard_bounds


def test_shard_bounds_cover_batch_once():
    for batch in (0, 1, 5, 7, 256, 1024):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def test_shard_bounds_reject_bad_rank():
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)
    with pytest.raises(ValueError):
        shard_bounds(-1, 2, 0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, batch, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        lo, hi = shard_bounds(batch, world, rank)
        # each problem's "value" is a function of its global index
        local = torch.arange(lo, hi, dtype=torch.float32) * 0.5 + 1.0
        full = gather_values(local, batch)
        q.put((rank, full.tolist()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world,batch", [(2, 6), (2, 5), (3, 7), (2, 1)])
def test_gather_values_gloo(world, batch):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, val = q.get(timeout=120)
            results[rank] = val
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    expect = [i * 0.5 + 1.0 for i in range(batch)]
    for r in range(world):
        assert results[r] == expect, results[r]
