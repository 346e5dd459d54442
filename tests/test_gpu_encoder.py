"""The prompt encoder (Qwen3-VL-8B's text model, ex-nihilo's encoder-states, src/encoder.lisp:143-183)
on the B200 against transformers' Qwen3VLTextModel (through tests/golden/encoder_small.npz) and the
oracle that restates it (oracle/encoder_oracle.py).

Tolerance: the projections take bf16 operands (the activations rounded once per GEMM; the weights
are the checkpoint's Q8_0 values rounded to bf16) with fp32 accumulation; the residual stream and
the embedding rows are fp32.  Two blocks are held to rel-L2 <= 2e-2, the DiT's per-block bound."""
import numpy as np
import pytest

import exn_b200 as E
from oracle import dit_oracle as O
from oracle import encoder_oracle as EO

pytestmark = pytest.mark.gpu
TOL = 2e-2
SMALL = dict(width=EO.SMALL.width, layers=EO.SMALL.layers, heads=EO.SMALL.heads, kv_heads=EO.SMALL.kv_heads,
             ffn=EO.SMALL.ffn, vocab=EO.SMALL.vocab)


@pytest.fixture(scope="module")
def small():
    e = E.Encoder(**SMALL)
    e.load_synthetic(1)
    yield e
    e.close()


@pytest.fixture(scope="module")
def small_wt():
    return EO.SynthEncoder(EO.SMALL, seed=1)


@pytest.mark.parametrize("case", ["text", "edit"])
def test_encoder_matches_transformers_golden(small, golden_dir, case):
    import os
    g = np.load(os.path.join(golden_dir, "encoder_small.npz"))
    ids, pos = g[case + "_ids"], g[case + "_positions"]
    got = small.states(ids, None if case == "text" else pos)
    err = O.rel_l2(got, g[case + "_states"])
    print("\nencoder %s prompt (%d tokens) against transformers: rel-L2 %.4g" % (case, len(ids), err))
    assert np.isfinite(got).all()
    assert err < TOL


@pytest.mark.parametrize("n", [1, 127, 300, 600])
def test_encoder_matches_oracle(small, small_wt, n):
    """Lengths around the attention's 128-row tiles and 64-key units (one token; one tile short of
    a row; three tiles, the last ragged), text positions; up to 512 tokens the GEMMs run split
    along K with the epilogues after the sum, 600 tokens take the fused epilogues."""
    ids = EO.synth_ids(EO.SMALL, n, seed=n)
    got = small.states(ids)
    want = EO.states(small_wt, EO.SMALL, ids)
    err = O.rel_l2(got, want)
    print("\nencoder %d tokens against the oracle: rel-L2 %.4g" % (n, err))
    assert err < TOL


def test_encoder_prefix_rows_do_not_see_later_tokens(small):
    """Causality: the first k tokens' states do not depend on the tokens after them."""
    ids = EO.synth_ids(EO.SMALL, 200, seed=9)
    a = small.states(ids)
    b = small.states(np.concatenate([ids[:150], (ids[150:] + 1) % EO.SMALL.vocab]))
    assert np.array_equal(a[:150], b[:150])
    assert not np.array_equal(a[150:], b[150:])


def test_encoder_is_deterministic(small):
    ids = EO.synth_ids(EO.SMALL, 77, seed=3)
    assert np.array_equal(small.states(ids), small.states(ids))


@pytest.mark.parametrize("mtype", ["q8_0", "bf16", "f32"])
def test_encoder_gguf_equals_synthetic(small, small_wt, tmp_path, mtype):
    """load-encoder's path: the same weights written as a qwen3vl GGUF (with a final norm the encoder
    does not read) load to the same bytes on the device, so the same states."""
    path = tmp_path / ("enc_%s.gguf" % mtype)
    EO.write_gguf(path, small_wt, matrix_type=mtype, extra=("output_norm.weight",))
    ids = EO.synth_ids(EO.SMALL, 64, seed=4)
    with E.load_encoder(path, **SMALL) as e:
        if mtype == "q8_0":
            assert e.weights_digest() == small.weights_digest()
            assert np.array_equal(E.encoder_states(e, ids), small.states(ids))
        elif mtype == "f32":
            # the dequantised values: the matrices round to the same bf16, the fp32 embedding table
            # holds the same values
            assert np.array_equal(e.states(ids), small.states(ids))
        else:
            # the dequantised values rounded to bf16: the same matrices, an embedding table rounded
            # once more (a bf16 rounding of every input row moves the states by ~1e-2, as much as
            # the bf16 operands of the whole pass)
            assert O.rel_l2(e.states(ids), small.states(ids)) < TOL


def test_encoder_gguf_errors(small_wt, tmp_path):
    """open-dit-style checks of the file (src/weights.lisp:47-61 for the DiT): architecture, missing
    tensors and wrong dims are named."""
    p1 = tmp_path / "arch.gguf"
    EO.write_gguf(p1, small_wt, arch="llama")
    p2 = tmp_path / "bad.gguf"
    EO.write_gguf(p2, small_wt, drop=("blk.1.ffn_up.weight",), bad_dims="blk.0.attn_k.weight")
    with E.Encoder(**SMALL) as e:
        with pytest.raises(E.ExnError) as x:
            e.load_gguf(p1)
        assert x.value.code == 3 and "architecture llama" in str(x.value)
        with pytest.raises(E.ExnError) as x:
            e.load_gguf(p2)
        assert x.value.code == 3
        assert "missing blk.1.ffn_up.weight" in str(x.value) and "blk.0.attn_k.weight is (480 256)" in str(x.value)
        assert not E.lib().exn_enc_weights_ready(e.h)
        with pytest.raises(E.ExnError) as x:
            e.states([1, 2, 3])
        assert x.value.code == 4


def test_encoder_rejects_bad_ids(small):
    with pytest.raises(E.ExnError) as x:
        small.states([0, EO.SMALL.vocab, 1])
    assert x.value.code == 1 and "token 1" in str(x.value)
    with pytest.raises(E.ExnError):
        small.states(np.zeros(0, dtype=np.int32))


def test_encoder_full_width_two_blocks_match_oracle():
    """Qwen3-VL-8B's block shape (width 4096, 32 / 8 heads, FFN 12288) with two blocks and a
    4096-token vocabulary, a 141-token prompt, against the oracle."""
    sh = EO.EncShape(layers=2, vocab=4096)
    wt = EO.SynthEncoder(sh, seed=1)
    ids = EO.synth_ids(sh, 141, seed=2)
    with E.Encoder(layers=2, vocab=4096) as e:
        e.load_synthetic(1)
        got = e.states(ids)
    want = EO.states(wt, sh, ids)
    err = O.rel_l2(got, want)
    print("\nencoder at full width, 2 blocks, 141 tokens: rel-L2 %.4g" % err)
    assert err < TOL


def test_encoder_full_model_prompt():
    """The whole 36-block model on a config-2 prompt's token count (the template's system turn,
    about 13 tokens, plus 128): finite states, and the device time of the pass."""
    with E.Encoder() as e:
        e.load_synthetic(1)
        ids = EO.synth_ids(EO.EncShape(), 141, seed=5)
        s = e.states(ids)
        ms = []
        for _ in range(3):
            e.states(ids)
            ms.append(e.last_ms())
    assert s.shape == (141, 4096) and np.isfinite(s).all()
    print("\nencoder, 36 blocks, 141 tokens: %.2f ms a prompt on the device (best of 3)" % min(ms))


def test_encoder_states_device_feed_the_dit():
    """encode-prompt to the DiT without the host: exn_enc_states_device writes the states after the
    system turn's rows into device memory, exn_generate_device reads them as its context, and the
    8-step latent is bit for bit the one the host path gives (states to host, then exn_generate)."""
    import torch
    enc_shape = dict(width=256, layers=2, heads=2, kv_heads=2, ffn=512, vocab=512)
    n, skip, h, w = 20, 4, 4, 6
    ids = EO.synth_ids(EO.EncShape(**enc_shape), n, seed=11)
    with E.Encoder(**enc_shape) as enc, E.Dit(width=256, layers=2, ffn=768, context=256) as dit:
        enc.load_synthetic(1)
        dit.load_synthetic(1)
        _, lat = O.synth_inputs(O.Shape(width=256, layers=2, ffn=768, context=256), n - skip, h, w, seed=3)
        z_host = dit.generate(enc.states(ids)[skip:], n - skip, lat[0], h, w)
        ctx_d = torch.full((n - skip, 256), float("nan"), dtype=torch.float32, device="cuda")
        enc.states_device(ids, ctx_d.data_ptr(), skip=skip)
        z_d = torch.from_numpy(np.ascontiguousarray(lat[0])).cuda()
        dit.generate_device(1, ctx_d.data_ptr(), n - skip, z_d.data_ptr(), h, w)
        torch.cuda.synchronize()
        assert np.array_equal(ctx_d.cpu().numpy(), enc.states(ids)[skip:])
        assert np.array_equal(z_d.cpu().numpy(), z_host)
        with pytest.raises(E.ExnError):
            enc.states_device(ids, ctx_d.data_ptr(), skip=n)

