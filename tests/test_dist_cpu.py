"""The multi-GPU host logic on CPU ranks (gloo, world size 2): shards of
pictures cover every picture exactly once, and the timing reduction is the
max over ranks, as bench.py uses them."""
import os
import socket

import pytest
import torch.multiprocessing as mp

import exn_dist as D


def test_shards_cover_once():
    for n in (1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            got = [i for r in range(world) for i in D.shard(n, r, world)]
            assert got == list(range(n))
            sizes = [len(D.shard(n, r, world)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1
    assert [list(b) for b in D.batches(range(3, 20), 8)] == [list(range(3, 11)), list(range(11, 19)), [19]]
    with pytest.raises(ValueError):
        D.shard(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = list(D.shard(64, rank, world))
        m = D.max_over_ranks(dist, 10.0 + rank)
        q.put((rank, mine, m))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0][1] + out[1][1] == list(range(64))
    assert out[0][2] == out[1][2] == 11.0
