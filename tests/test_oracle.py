"""The oracle (oracle/dit_oracle.py) held to the golden vectors that the
reference's own inspect/ref_dit.py produced (tests/golden/make_golden.py)."""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import dit_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(case):
    path = os.path.join(GOLDEN, case + ".npz")
    if not os.path.exists(path):
        pytest.skip("golden %s not generated" % case)
    g = np.load(path)
    return g, json.loads(str(g["meta"]))


def _digest(sw):
    h = hashlib.sha256()
    for name, _ in O.expected_tensors(sw.shape):
        if name in sw.vec:
            h.update(sw.vec[name].tobytes())
        else:
            qs, d = sw.q8[name]
            h.update(qs.tobytes())
            h.update(d.tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("case", ["tiny", "cfg1"])
def test_forward_matches_ref_dit(case):
    g, m = _load(case)
    sh = O.Shape(**m["shape"])
    sw = O.SynthWeights.make(sh, seed=m["weight_seed"])
    assert _digest(sw) == str(g["weights_sha256"]), "synthetic generator drifted"
    ctx, lat = O.synth_inputs(sh, m["p"], m["h"], m["w"], seed=m["input_seed"])
    assert hashlib.sha256(ctx[0].tobytes()).hexdigest() == str(g["ctx_sha256"])
    assert hashlib.sha256(lat[0].tobytes()).hexdigest() == str(g["lat_sha256"])
    trace = []
    v = O.forward(sw, sh, ctx[0], lat[0], m["sigma"], trace=trace)
    # the fp32 ladder's bar (docs/design.md:241-243): cosine 1, max diff ~1e-5
    assert O.rel_l2(trace[0], g["txt"]) < 1e-5
    assert O.rel_l2(trace[1][g["blk0_rows"]], g["blk0"]) < 1e-5
    assert O.rel_l2(v, g["v"]) < 1e-5
    rms = [float(np.sqrt((x.astype(np.float64) ** 2).mean())) for x in trace[1:]]
    np.testing.assert_allclose(rms, g["block_rms"], rtol=1e-3)


@pytest.mark.parametrize("case", ["tiny_euler", "small_euler"])
def test_euler_matches_ref_dit(case):
    g, m = _load(case)
    sh = O.Shape(**m["shape"])
    sw = O.SynthWeights.make(sh, seed=m["weight_seed"])
    ctx, lat = O.synth_inputs(sh, m["p"], m["h"], m["w"], seed=m["input_seed"])
    vs = []
    z = O.euler(sw, sh, ctx[0], lat[0], velocities=vs)
    assert O.rel_l2(vs[0], g["v_first"]) < 1e-5
    assert O.rel_l2(z, g["z"]) < 1e-5


def test_q8_0_matches_gguf_py():
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((64, 256)) * rng.uniform(0.001, 3, (64, 1))).astype(np.float32)
    x[3, :32] = 0          # an all-zero block: d = 0
    x[5, 7] = 1e-30        # tiny values
    qs, d = O.q8_0_quantize(x)
    ref = quants.quantize(x, gguf.GGMLQuantizationType.Q8_0)
    mine = O.q8_0_pack(qs, d).reshape(ref.shape)
    assert np.array_equal(mine, ref)
    back = quants.dequantize(ref, gguf.GGMLQuantizationType.Q8_0)
    assert np.array_equal(O.q8_0_dequantize(qs, d), back)


def test_schema_counts():
    # 9 + 32 x 8 = 265 tensors (src/weights.lisp:22-45)
    assert len(O.expected_tensors(O.Shape())) == 265


def test_positions_plain():
    # ref_dit.py:62-69 / host.lisp:32-44: text (i,i,i), image at frame P centred
    pos = O.dit_positions(3, 2, 3)
    assert pos[:3] == [(0, 0, 0), (1, 1, 1), (2, 2, 2)]
    assert pos[3:] == [(3, -1, -2), (3, -1, -1), (3, -1, 0), (3, 0, -2), (3, 0, -1), (3, 0, 0)]


def test_positions_edit():
    # host.lisp:43-50 with REF (A=2, RH=1, RW=2), P = 5 prefix rows (2 text, 2 ref, 1 text)
    pos = O.dit_positions(5, 1, 1, (2, 1, 2))
    assert pos[:2] == [(0, 0, 0), (1, 1, 1)]
    assert pos[2:4] == [(2, -1, -1), (2, -1, 0)]          # the reference block at frame A
    assert pos[4] == (4, 4, 4)                            # text resumes at A + max(RH, RW)
    assert pos[5] == (5, -1, -1)                          # the target after it


def test_mask_cases():
    # dit.cu:64-66: image rows see all L keys; B0..B1-1 see their block; else causal
    p, l, b0, b1 = 40, 100, 12, 30
    g = np.arange(60)
    lim = O.xa_lim(g, p, l, b0, b1)
    assert lim[5] == 5 and lim[12] == 29 and lim[29] == 29 and lim[30] == 30 and lim[45] == 99
    assert np.all(np.diff(lim) >= 0)   # never decreasing: a tile's last key is its last row's


def test_synth_generator_stats():
    u = O.synth_normal(1, 7, (1 << 16,), 1.0)
    assert abs(float(u.mean())) < 0.02 and abs(float(u.std()) - 1.0) < 0.02


def test_vae_oracle_matches_ref_vae_golden(golden_dir):
    """oracle/vae_oracle.py against the reference's own inspect/ref_vae.py (tests/golden/vae_small.npz:
    the oracle's synthetic decoder written as a BF16 safetensors file, an 8 x 8 latent, 128 x 128
    RGBA out): the same fp32 arithmetic, so rel-L2 < 1e-5."""
    import hashlib
    from oracle import vae_oracle as V
    g = np.load(os.path.join(golden_dir, "vae_small.npz"))
    sw = V.SynthVae(1)
    z = O.synth_normal(0, 3000, (64, 8, 8))
    assert hashlib.sha256(z.tobytes()).hexdigest() == str(g["latent_sha256"])
    out = V.decode(sw, z)
    assert out.shape == (4, 128, 128)
    assert O.rel_l2(out, g["rgba"]) < 1e-5


@pytest.mark.parametrize("case", ["text", "edit"])
def test_encoder_oracle_matches_transformers_golden(golden_dir, case):
    """oracle/encoder_oracle.py against transformers' Qwen3VLTextModel (tests/golden/encoder_small.npz,
    made by make_encoder_golden.py with the oracle's synthetic weights): the last block's output before
    the final norm, for text positions and an edit prompt's M-RoPE positions; fp32 both, rel-L2 < 1e-5."""
    from oracle import encoder_oracle as EO
    g = np.load(os.path.join(golden_dir, "encoder_small.npz"))
    wt = EO.SynthEncoder(EO.SMALL, seed=1)
    ids = g[case + "_ids"]
    assert np.array_equal(ids, EO.synth_ids(EO.SMALL, len(ids), seed={"text": 0, "edit": 1}[case]))
    pos = g[case + "_positions"]
    want = EO.text_positions(len(ids)) if case == "text" else EO.edit_positions(6, 3, 5, 9)
    assert np.array_equal(pos, want)
    got = EO.states(wt, EO.SMALL, ids, pos)
    assert O.rel_l2(got, g[case + "_states"]) < 1e-5


def test_encoder_mrope_rule():
    """mrope-table (src/encoder.lisp:26-39): frequency j turns by h where j mod 3 is 1 and by w where it
    is 2, below 60; by t elsewhere.  For (i, i, i) it is plain RoPE at position i."""
    from oracle import encoder_oracle as EO
    a = EO.mrope_angles(EO.SMALL, np.array([[7, 100, 1000]]))[0]
    inv = 5e6 ** (-(2.0 * np.arange(64)) / 128)
    for j in range(64):
        want = (1000 if j % 3 == 2 else 100 if j % 3 == 1 else 7) if j < 60 else 7
        assert a[j] == want * inv[j]
    t = EO.mrope_angles(EO.SMALL, EO.text_positions(5))
    assert np.allclose(t, np.arange(5)[:, None] * inv[None, :], rtol=0, atol=0)
