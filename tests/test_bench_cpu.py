"""Host-side logic of bench.py's multi-GPU path, on CPU with gloo ranks:
utterance sharding (disjoint, covering) and the max-over-ranks timing."""
import os
import socket

import pytest
import torch.multiprocessing as mp

import bench


def test_shard_disjoint_cover():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            seen += list(bench.shard(64 * world, r, world))
        assert sorted(seen) == list(range(64 * world))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        out = bench.max_over_ranks([1.0 + rank, 10.0 - rank], world, device="cpu")
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r] == [2.0, 10.0]
