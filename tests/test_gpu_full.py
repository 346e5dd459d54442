"""The full-size DiT (D=4096, 32 blocks, 1024^2 = 64 x 64 latent, 128 text
rows) on the B200: the 8-step latent against the
reference's own ref_dit.py (tests/golden/cfg2_euler.npz, cosine >= 0.999)
and size-independent properties (cached prefix == recomputed prefix; a
batch == its pictures one by one)."""
import json
import os

import numpy as np
import pytest

import exn_b200 as E
from oracle import dit_oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "cfg2_euler.npz")
P, H, W = 128, 64, 64


@pytest.fixture(scope="module")
def full():
    d = E.Dit()
    d.load_synthetic(1)
    yield d
    d.close()


@pytest.fixture(scope="module")
def inputs():
    return O.synth_inputs(O.Shape(), P, H, W, seed=0, batch=2)


def test_full_eight_steps_match_ref_dit(full, inputs):
    if not os.path.exists(GOLDEN):
        pytest.fail("tests/golden/cfg2_euler.npz missing")
    g = np.load(GOLDEN)
    ctx, lat = inputs
    z = full.generate(ctx[0], P, lat[0], H, W, O.TURBO_SIGMAS, prefix_key="cfg2")
    assert np.isfinite(z).all()
    assert O.cosine(z, g["z"]) >= 0.999
    assert O.rel_l2(z, g["z"]) < 2e-2


def test_full_cached_prefix_equals_recomputed(full, inputs):
    ctx, lat = inputs
    full.velocity(ctx[1], P, lat[1], H, W, 1.0, prefix_key="p1")
    a = full.velocity(ctx[1], P, lat[1], H, W, 0.5, prefix_key="p1")
    b = full.velocity(ctx[1], P, lat[1], H, W, 0.5)
    assert O.rel_l2(a, b) < 1e-6


def test_full_batch_equals_single(full, inputs):
    ctx, lat = inputs
    zb = full.generate_batch(ctx, P, lat, H, W)
    for i in range(2):
        zi = full.generate(ctx[i], P, lat[i], H, W, prefix_key=("one", i))
        assert O.rel_l2(zb[i], zi) < 1e-6
