"""The whole DiT step and Euler loop on the B200 against the oracle and the
golden vectors that the reference's own inspect/ref_dit.py produced.

Tolerances: per-block activations rel-L2 <= 2e-2, the
8-step latent cosine >= 0.999; bf16 tensor-core operands, fp32 accumulation,
fp32 residual stream.  A block's residual update is also checked on its own
(rel-L2 of x_after - x_before <= 2e-2), so a small gate cannot hide it."""
import json
import os

import numpy as np
import pytest

import exn_b200 as E
from oracle import dit_oracle as O
from oracle.synth_gguf import write_gguf

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TINY = dict(width=256, layers=2, ffn=768, context=256)
SMALL = dict(width=512, layers=3, ffn=1536, context=512)
TOL = 2e-2


def golden(case):
    g = np.load(os.path.join(GOLDEN, case + ".npz"))
    return g, json.loads(str(g["meta"]))


@pytest.fixture(scope="module")
def tiny():
    d = E.Dit(**TINY)
    d.load_synthetic(1)
    yield d
    d.close()


@pytest.fixture(scope="module")
def tiny_sw():
    return O.SynthWeights.make(O.Shape(**TINY), seed=1)


def test_tiny_blocks_match_oracle(tiny, tiny_sw):
    sh = O.Shape(**TINY)
    p, h, w, sigma = 8, 4, 6, 0.7
    ctx, lat = O.synth_inputs(sh, p, h, w)
    ctx, lat = ctx[0], lat[0]
    n = p + h * w
    trace = np.zeros((sh.layers + 1, n, sh.width), dtype=np.float32)
    tiny._ck(E.lib().exn_test_trace(tiny.h, trace.ctypes.data, trace.size))
    try:
        v = tiny.velocity(ctx, p, lat, h, w, sigma)
    finally:
        tiny._ck(E.lib().exn_test_trace(tiny.h, None, 0))
    want_tr = []
    want_v = O.forward(tiny_sw, sh, ctx, lat, sigma, trace=want_tr)
    assert O.rel_l2(trace[0][:p], want_tr[0]) < TOL
    x_prev_g, x_prev_w = trace[0], None
    for i in range(sh.layers):
        xg, xw = trace[i + 1], want_tr[i + 1]
        assert O.rel_l2(xg, xw) < TOL, i
        if i > 0:
            assert O.rel_l2(xg - trace[i], xw - want_tr[i]) < TOL, i
    assert O.rel_l2(v, want_v) < TOL


@pytest.mark.parametrize("case", ["tiny", "cfg1"])
def test_velocity_matches_ref_dit_golden(case):
    g, m = golden(case)
    sh = O.Shape(**m["shape"])
    ctx, lat = O.synth_inputs(sh, m["p"], m["h"], m["w"], seed=m["input_seed"])
    with E.Dit(**m["shape"]) as d:
        d.load_synthetic(m["weight_seed"])
        n = m["p"] + m["h"] * m["w"]
        trace = np.zeros((sh.layers + 1, n, sh.width), dtype=np.float32)
        d._ck(E.lib().exn_test_trace(d.h, trace.ctypes.data, trace.size))
        v = d.velocity(ctx[0], m["p"], lat[0], m["h"], m["w"], m["sigma"])
        d._ck(E.lib().exn_test_trace(d.h, None, 0))
    assert O.rel_l2(trace[0][:m["p"]], g["txt"]) < TOL
    assert O.rel_l2(trace[1][g["blk0_rows"]], g["blk0"]) < TOL
    assert O.rel_l2(trace[1][g["blk0_rows"]] - trace[0][g["blk0_rows"]],
                    g["blk0"] - np.concatenate([g["txt"], trace[0][m["p"]:]])[g["blk0_rows"]]) < 5e-2
    assert O.rel_l2(v, g["v"]) < TOL


@pytest.mark.parametrize("case", ["tiny_euler", "small_euler"])
def test_eight_steps_match_ref_dit_golden(case):
    g, m = golden(case)
    sh = O.Shape(**m["shape"])
    ctx, lat = O.synth_inputs(sh, m["p"], m["h"], m["w"], seed=m["input_seed"])
    with E.Dit(**m["shape"]) as d:
        d.load_synthetic(m["weight_seed"])
        z = d.generate(ctx[0], m["p"], lat[0], m["h"], m["w"], O.TURBO_SIGMAS, prefix_key="prompt")
    assert O.cosine(z, g["z"]) >= 0.999
    assert O.rel_l2(z, g["z"]) < TOL


def test_prefix_cache_is_exact(tiny):
    sh = O.Shape(**TINY)
    p, h, w = 8, 4, 6
    ctx, lat = O.synth_inputs(sh, p, h, w, seed=5)
    tiny.velocity(ctx[0], p, lat[0], h, w, 1.0, prefix_key="k1")          # first pass keeps the prompt K/V
    v_cached = tiny.velocity(ctx[0], p, lat[0] * 0.5, h, w, 0.9, prefix_key="k1")
    v_full = tiny.velocity(ctx[0], p, lat[0] * 0.5, h, w, 0.9)             # no key: the joint sequence again
    assert O.rel_l2(v_cached, v_full) < 1e-6
    # another prompt under the same key length must not reuse the kept rows
    v_other = tiny.velocity(ctx[0] * -1, p, lat[0] * 0.5, h, w, 0.9, prefix_key="k2")
    assert O.rel_l2(v_other, v_full) > 1e-3


def test_generate_matches_velocity_loop(tiny):
    sh = O.Shape(**TINY)
    p, h, w = 8, 4, 6
    ctx, lat = O.synth_inputs(sh, p, h, w, seed=9)
    z = lat[0].copy()
    for s, s2 in zip(O.TURBO_SIGMAS[:-1], O.TURBO_SIGMAS[1:]):
        z = z + np.float32(s2 - s) * tiny.velocity(ctx[0], p, z, h, w, s, prefix_key="loop")
    zf = tiny.generate(ctx[0], p, lat[0], h, w, O.TURBO_SIGMAS, prefix_key="fused")
    assert O.rel_l2(zf, z) < 1e-6


def test_edit_reference_matches_oracle(tiny, tiny_sw):
    sh = O.Shape(**TINY)
    p, h, w = 10, 4, 4
    a, rh, rw = 3, 3, 5
    ctx, lat = O.synth_inputs(sh, p, h, w, seed=11)
    _, rlat = O.synth_inputs(sh, 1, rh, rw, seed=12)
    v = tiny.velocity(ctx[0], p, lat[0], h, w, 0.8, prefix_key=("edit", 1), ref=(a, rlat[0], rh, rw))
    want = O.forward(tiny_sw, sh, ctx[0], lat[0], 0.8, ref=(a, rlat[0]))
    assert O.rel_l2(v, want) < TOL
    # the cached second step against the oracle
    v2 = tiny.velocity(ctx[0], p, lat[0] * 0.7, h, w, 0.6, prefix_key=("edit", 1), ref=(a, rlat[0], rh, rw))
    want2 = O.forward(tiny_sw, sh, ctx[0], lat[0] * 0.7, 0.6, ref=(a, rlat[0]))
    assert O.rel_l2(v2, want2) < TOL


def test_last_call_time_is_the_device_part(tiny):
    # the device time of a host-buffer call: positive and within the call's own wall clock
    import time
    sh = O.Shape(**TINY)
    p, h, w = 8, 4, 6
    ctx, lat = O.synth_inputs(sh, p, h, w, seed=31)
    t0 = time.perf_counter()
    tiny.generate(ctx[0], p, lat[0], h, w)
    wall_ms = (time.perf_counter() - t0) * 1e3
    ms = tiny.last_call_ms()
    assert 0.0 < ms <= wall_ms


def test_batch_equals_single(tiny):
    sh = O.Shape(**TINY)
    p, h, w, b = 8, 4, 6, 3
    ctx, lat = O.synth_inputs(sh, p, h, w, seed=21, batch=b)
    zb = tiny.generate_batch(ctx, p, lat, h, w)
    for i in range(b):
        zi = tiny.generate(ctx[i], p, lat[i], h, w, prefix_key=("single", i))
        assert O.rel_l2(zb[i], zi) < 1e-6, i


@pytest.mark.parametrize("mtype", ["q8_0", "f32", "bf16", "f16"])
def test_gguf_upload_equals_synthetic(tmp_path, tiny, tiny_sw, mtype):
    path = tmp_path / "dit.gguf"
    write_gguf(path, tiny_sw, matrix_type=mtype)
    sh = O.Shape(**TINY)
    p, h, w = 8, 4, 6
    ctx, lat = O.synth_inputs(sh, p, h, w, seed=2)
    d = E.upload_dit(path, **TINY)
    try:
        v = E.dit_velocity(d, ctx[0], p, lat[0], h, w, 0.5)
    finally:
        E.dit_release(d)
        d.close()
    v0 = tiny.velocity(ctx[0], p, lat[0], h, w, 0.5)
    if mtype == "q8_0":
        assert O.rel_l2(v, v0) < 1e-6
    elif mtype == "f32":   # f32 holds q * d exactly: only the GEMVs' order of summation differs
        assert O.rel_l2(v, v0) < 5e-3
    else:   # the GEMV matrices (timestep MLP, modulation) keep the f16- or bf16-rounded values
        assert O.rel_l2(v, v0) < 1e-2


@pytest.mark.parametrize("mtype", ["f32", "bf16", "f16"])
def test_gguf_gemm_matrix_conversion_is_exact(tmp_path, tiny_sw, mtype):
    """A GEMM matrix stored as f32 / bf16 / f16 lands in the bf16 slab as the round-to-nearest bf16
    of the stored value, bit for bit (f16 widens to f32 exactly first)."""
    import torch
    path = tmp_path / "dit.gguf"
    write_gguf(path, tiny_sw, matrix_type=mtype)
    name = "transformer_blocks.1.img_mlp.gate_up.weight"   # interleaved on the device: undone by the reader
    qs, dq = tiny_sw.q8[name]
    vals = O.q8_0_dequantize(qs, dq)
    if mtype == "f16":
        vals = vals.astype(np.float16).astype(np.float32)
    want = torch.from_numpy(np.ascontiguousarray(vals)).to(torch.bfloat16).view(torch.int16).numpy()
    d = E.upload_dit(path, **TINY)
    try:
        got = np.empty(want.shape, dtype=np.int16)
        d._ck(E.lib().exn_test_weight_bf16(d.h, name.encode(), got.ctypes.data, got.size))
    finally:
        d.close()
    assert np.array_equal(got, want)


def test_errors_are_reported():
    with E.Dit(**TINY) as d:
        sh = O.Shape(**TINY)
        ctx, lat = O.synth_inputs(sh, 4, 2, 2)
        with pytest.raises(E.ExnError) as e:
            d.velocity(ctx[0], 4, lat[0], 2, 2, 0.5)
        assert e.value.code == 4          # no weights yet
        d.load_synthetic(1)
        with pytest.raises(E.ExnError) as e:
            d.load_tensor("img_in.weight", E.GGML_F32, (64, 128), np.zeros((128, 64), np.float32))
        assert e.value.code == 3 and "not (64 256)" in str(e.value)
        with pytest.raises(E.ExnError):
            d.velocity(ctx[0], 4, lat[0], 2, 2, 0.5, ref=(9, lat[0], 2, 2))   # A past the prompt
        d.velocity(ctx[0], 4, lat[0], 2, 2, 0.5)                            # still usable
