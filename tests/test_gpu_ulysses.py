"""Sequence parallelism (Ulysses) over 2 (and, where there are 4 or 8, 4 and 8) GPUs: the rows of one
picture split between the processes, Q/K/V and the attention output stored by the QKV GEMM and
the attention kernel straight into the rank that keeps them (peer memory over NVLink).  Every
row's arithmetic is the one-GPU arithmetic, so the result must equal a one-GPU handle's bit for
bit (rel-L2 < 1e-6): plain and edit layouts, the first pass and a cached one, the fused 8-step
loop.  NVLS off (a rank's failure must not leave NVLink multicast state)."""
import os
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
SHAPE = dict(width=512, layers=2, ffn=1536, context=512)


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _two_gpus():
    return _gpus() >= 2


# world size -> (DiT shape, reference picture h, w): width / world a multiple of 256, and the
# prefix (8 text rows + the reference's) and image (4 x 6) rows divisible by the world size
CASES = {2: (SHAPE, 2, 3), 4: (dict(width=1024, layers=2, ffn=3072, context=512), 2, 2),
         8: (dict(width=2048, layers=2, ffn=6144, context=512), 2, 4)}


def _rank(rank, world, uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import exn_b200 as E
        from oracle import dit_oracle as O
        shape, rh, rw = CASES[world]
        sh = O.Shape(**shape)
        out = {}
        with E.Dit(device=rank, **shape) as d:
            d.load_synthetic(1)
            d.comm_init(uid, rank, world)
            p, h, w = 8, 4, 6
            ctx, lat = O.synth_inputs(sh, p, h, w, seed=3)
            out["v1"] = d.velocity(ctx[0], p, lat[0], h, w, 0.9, prefix_key="k")
            out["v2"] = d.velocity(ctx[0], p, lat[0] * 0.5, h, w, 0.7, prefix_key="k")     # cached prefix
            out["z"] = d.generate(ctx[0], p, lat[0], h, w, prefix_key="g")
            _, rl = O.synth_inputs(sh, 1, rh, rw, seed=4)
            out["ve"] = d.velocity(ctx[0], p, lat[0], h, w, 0.8, prefix_key=("e", 1), ref=(2, rl[0], rh, rw))
        q.put((rank, out, None))
    except Exception:
        q.put((rank, None, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sequence_parallel_equals_one_gpu(world):
    if _gpus() < world:
        pytest.skip("needs %d GPUs" % world)
    import torch.multiprocessing as mp
    import exn_b200 as E
    from oracle import dit_oracle as O
    uid = E.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = {}
    for _ in procs:
        r, out, err = q.get(timeout=300)
        assert err is None, err
        res[r] = out
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    shape, rh, rw = CASES[world]
    sh = O.Shape(**shape)
    p, h, w = 8, 4, 6
    c, lat = O.synth_inputs(sh, p, h, w, seed=3)
    _, rl = O.synth_inputs(sh, 1, rh, rw, seed=4)
    with E.Dit(device=0, **shape) as d:
        d.load_synthetic(1)
        want = {"v1": d.velocity(c[0], p, lat[0], h, w, 0.9, prefix_key="k"),
                "v2": d.velocity(c[0], p, lat[0] * 0.5, h, w, 0.7, prefix_key="k"),
                "z": d.generate(c[0], p, lat[0], h, w, prefix_key="g"),
                "ve": d.velocity(c[0], p, lat[0], h, w, 0.8, prefix_key=("e", 1), ref=(2, rl[0], rh, rw))}
    for key, v in want.items():
        for r in range(world):
            assert O.rel_l2(res[r][key], v) < 1e-6, (key, r, O.rel_l2(res[r][key], v))


def _lonely(uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["EXN_COMM_TIMEOUT_S"] = "3"
    try:
        import time
        import exn_b200 as E
        with E.Dit(device=0, **SHAPE) as d:
            t0 = time.time()
            try:
                d.comm_init(uid, 0, 2)          # rank 1 never joins
                q.put(("joined", 0.0))
            except E.ExnError as e:
                q.put((e.code, time.time() - t0))
    except Exception:
        q.put((traceback.format_exc(), 0.0))


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_missing_rank_times_out_on_the_host():
    import torch.multiprocessing as mp
    import exn_b200 as E
    uid = E.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    pr = ctx.Process(target=_lonely, args=(uid, q))
    pr.start()
    code, dt = q.get(timeout=120)
    pr.join(timeout=60)
    assert code == 6, code          # EXN_ETIMEOUT
    assert dt < 30
