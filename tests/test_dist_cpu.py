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


def _sp_worker(rank, world, port, q, with_ref):
    import numpy as np
    import torch
    import torch.distributed as dist
    from oracle import dit_oracle as O
    from oracle import ulysses_model as U
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = O.Shape(width=256, layers=2, ffn=768, context=256)
        sw = O.SynthWeights.make(sh, seed=1)
        ctx, lat = O.synth_inputs(sh, 8, 4, 6, seed=3)
        ref = None
        if with_ref:
            _, rl = O.synth_inputs(sh, 1, 2, 3, seed=4)
            ref = (2, rl[0])

        def all_to_all(chunks):
            shape = chunks[0].shape
            src = torch.from_numpy(np.concatenate(chunks).ravel())
            dst = torch.empty_like(src)
            dist.all_to_all_single(dst, src)
            return [a.reshape(shape) for a in np.split(dst.numpy(), world)]

        v = U.forward_rank(sw, sh, ctx[0], lat[0], 0.8, rank, world, all_to_all, ref=ref)
        q.put((rank, v))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("with_ref", [False, True])
def test_sequence_parallel_sharding_on_gloo_ranks(with_ref):
    """The library's Ulysses partitioning (rows per rank, head-group all-to-all) on two CPU ranks
    reproduces the unsharded oracle forward."""
    import numpy as np
    from oracle import dit_oracle as O
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sp_worker, args=(r, 2, port, q, with_ref)) for r in range(2)]
    for p in procs:
        p.start()
    parts = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    sh = O.Shape(width=256, layers=2, ffn=768, context=256)
    sw = O.SynthWeights.make(sh, seed=1)
    c, lat = O.synth_inputs(sh, 8, 4, 6, seed=3)
    ref = None
    if with_ref:
        _, rl = O.synth_inputs(sh, 1, 2, 3, seed=4)
        ref = (2, rl[0])
    want = O.forward(sw, sh, c[0], lat[0], 0.8, ref=ref).reshape(64, 24)
    got = np.concatenate([parts[0], parts[1]], axis=1)
    assert O.rel_l2(got, want) < 1e-5
