"""Host-side logic of bench.py's multi-GPU path, on CPU with gloo ranks:
utterance sharding (disjoint, covering), each rank's workload (exactly its
shard's prompts, in batch order) and the max-over-ranks timing."""
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


def _digest(utt):
    import hashlib

    ids, prompt = utt
    return hashlib.sha256(ids.tobytes() + prompt.tobytes()).hexdigest()


def _workload_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = [_digest(u) for u in bench.rank_workload(rank, world, vocab=32000)]
        every = [None] * world
        dist.all_gather_object(every, mine)
        q.put((rank, mine, every))
    finally:
        dist.destroy_process_group()


def test_rank_workloads_gloo():
    """world 2 on gloo: each rank decodes exactly its contiguous shard of the
    128-utterance batch (64 each, batch order), the shards are disjoint and
    cover the batch, and every rank sees the same assignment."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_workload_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r: (mine, every) for r, mine, every in (q.get(timeout=120) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    batch = [_digest(u) for u in bench.utterances(bench.B_PER_GPU * world, seed=3, vocab=32000)]
    for r in range(world):
        mine, every = res[r]
        assert mine == batch[r * bench.B_PER_GPU:(r + 1) * bench.B_PER_GPU]
        assert every == [res[k][0] for k in range(world)]
    assert sorted(res[0][0] + res[1][0]) == sorted(batch)
    assert not set(res[0][0]) & set(res[1][0])
