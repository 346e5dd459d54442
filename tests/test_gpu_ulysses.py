"""Sequence parallelism (Ulysses) over 2 GPUs: the rows of one picture split
between two processes, Q/K/V and the attention output exchanged by NCCL
all-to-all.  Every row's arithmetic is the one-GPU arithmetic, so the result
must equal a one-GPU handle's bit for bit (rel-L2 < 1e-6): plain and edit
layouts, the first pass and a cached one, the fused 8-step loop.  Needs two
GPUs; NVLS off (a rank's failure must not leave NVLink multicast state)."""
import os
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
SHAPE = dict(width=512, layers=2, ffn=1536, context=512)


def _two_gpus():
    try:
        import torch
        return torch.cuda.device_count() >= 2
    except Exception:
        return False


def _rank(rank, world, uid, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import exn_b200 as E
        from oracle import dit_oracle as O
        sh = O.Shape(**SHAPE)
        out = {}
        with E.Dit(device=rank, **SHAPE) as d:
            d.load_synthetic(1)
            d.comm_init(uid, rank, world)
            p, h, w = 8, 4, 6
            ctx, lat = O.synth_inputs(sh, p, h, w, seed=3)
            out["v1"] = d.velocity(ctx[0], p, lat[0], h, w, 0.9, prefix_key="k")
            out["v2"] = d.velocity(ctx[0], p, lat[0] * 0.5, h, w, 0.7, prefix_key="k")     # cached prefix
            out["z"] = d.generate(ctx[0], p, lat[0], h, w, prefix_key="g")
            _, rl = O.synth_inputs(sh, 1, 2, 3, seed=4)
            out["ve"] = d.velocity(ctx[0], p, lat[0], h, w, 0.8, prefix_key=("e", 1), ref=(2, rl[0], 2, 3))
        q.put((rank, out, None))
    except Exception:
        q.put((rank, None, traceback.format_exc()))


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
def test_two_rank_sequence_parallel_equals_one_gpu():
    import torch.multiprocessing as mp
    import exn_b200 as E
    from oracle import dit_oracle as O
    uid = E.comm_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, q)) for r in range(2)]
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
    sh = O.Shape(**SHAPE)
    p, h, w = 8, 4, 6
    c, lat = O.synth_inputs(sh, p, h, w, seed=3)
    _, rl = O.synth_inputs(sh, 1, 2, 3, seed=4)
    with E.Dit(device=0, **SHAPE) as d:
        d.load_synthetic(1)
        want = {"v1": d.velocity(c[0], p, lat[0], h, w, 0.9, prefix_key="k"),
                "v2": d.velocity(c[0], p, lat[0] * 0.5, h, w, 0.7, prefix_key="k"),
                "z": d.generate(c[0], p, lat[0], h, w, prefix_key="g"),
                "ve": d.velocity(c[0], p, lat[0], h, w, 0.8, prefix_key=("e", 1), ref=(2, rl[0], 2, 3))}
    for key, v in want.items():
        for r in (0, 1):
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
