"""The VAE decoder (Wan 2.2's, one frame: the step after the DiT, src/cuda-vae.lisp:94-136) on the
B200 against the reference's own numpy decoder (inspect/ref_vae.py, through tests/golden/vae_small.npz)
and the oracle that restates it (oracle/vae_oracle.py).

Tolerance: the convolutions take bf16 operands (the activations rounded once per convolution; the
weights are the checkpoint's bf16 exactly) with fp32 accumulation, the stream between them stays fp32;
about 30 such convolutions and an attention stand between the latent and the picture, so the RGBA
picture is held to rel-L2 <= 2e-2, the DiT's per-block bound."""
import numpy as np
import pytest

import exn_b200 as E
from oracle import dit_oracle as O
from oracle import vae_oracle as V

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def vae():
    v = E.Vae()
    v.load_synthetic(1)
    yield v
    v.close()


def _latent(h, w, seed=0):
    return O.synth_normal(seed, 3000, (64, h, w))


def test_vae_matches_ref_vae_golden(vae, golden_dir):
    import os
    g = np.load(os.path.join(golden_dir, "vae_small.npz"))
    rgba = vae.decode(_latent(8, 8), 8, 8)            # 128 x 128 x 4, channels last
    got = rgba.transpose(2, 0, 1)
    err = O.rel_l2(got, g["rgba"])
    print("\nVAE 8 x 8 latent against ref_vae.py: rel-L2 %.4g, max |diff| %.4g" % (err, np.abs(got - g["rgba"]).max()))
    assert np.isfinite(got).all()
    assert err < TOL


@pytest.mark.parametrize("h,w", [(8, 24), (16, 32)])
def test_vae_non_square_matches_oracle(vae, h, w):
    """Non-square latents against the fp32 oracle.  8 x 24 (a 128 x 384 picture): widths 24, 48,
    96, 192, 384 through the stages, none of the first four dividing 128 nor a multiple of it (the
    pixel tiles are 8, 16, 32, 64 columns wide, the 8-wide ones taller than the picture), like config
    3's 96-wide latent; 16 x 32 (a 256 x 512 picture): tiles of whole rows, then row segments."""
    z = _latent(h, w, seed=5)
    got = vae.decode(z, h, w).transpose(2, 0, 1)
    want = V.decode(V.SynthVae(1), z)
    err = O.rel_l2(got, want)
    print("\nVAE %d x %d latent against the oracle: rel-L2 %.4g" % (h, w, err))
    assert err < TOL


def test_vae_safetensors_equals_synthetic(vae, tmp_path):
    """upload-vae's path: the same weights written as a BF16 safetensors file (with an unused extra
    tensor, as a checkpoint holds the encoder too), checked and uploaded, decode the same bits."""
    sw = V.SynthVae(1)
    path = tmp_path / "vae.safetensors"
    V.write_safetensors(path, [(n, sw(n)) for n, _ in sw.spec] + [("encoder.conv1.bias", np.zeros(96, np.float32))])
    z = _latent(8, 8, seed=2)
    want = vae.decode(z, 8, 8)
    v2 = E.upload_vae(path)
    try:
        got = E.vae_decode(v2, z, 8, 8)
    finally:
        E.vae_release(v2)
        v2.close()
    assert np.array_equal(got, want)


def test_vae_safetensors_shape_errors(tmp_path):
    """open-vae's checks (src/weights.lisp:116-127): a missing tensor and a wrong shape are named."""
    sw = V.SynthVae(1)
    tensors = [(n, sw(n)) for n, _ in sw.spec if n != "decoder.head.2.bias"]
    tensors = [(n, np.zeros((32,), np.float32)) if n == "conv2.bias" else (n, a) for n, a in tensors]
    path = tmp_path / "bad.safetensors"
    V.write_safetensors(path, tensors)
    with E.Vae() as v:
        with pytest.raises(E.ExnError) as e:
            v.load_safetensors(path)
        assert e.value.code == 3
        assert "missing decoder.head.2.bias" in str(e.value) and "conv2.bias is (32), not (64)" in str(e.value)


def test_vae_full_picture(vae):
    """BASELINE config 2's picture: a 64 x 64 latent to 1024 x 1024 RGBA, finite and in -1 .. 1."""
    rgba = vae.decode(_latent(64, 64, seed=7), 64, 64)
    assert rgba.shape == (1024, 1024, 4)
    assert np.isfinite(rgba).all() and rgba.min() >= -1 and rgba.max() <= 1
    assert rgba.std() > 1e-3
    print("\nVAE 64 x 64 latent: %.2f ms on the device" % vae.last_ms())


def test_vae_rejects_unsupported_sizes(vae):
    # the middle attention takes the latent's pixels 64 at a time
    with pytest.raises(E.ExnError) as e:
        vae.decode(_latent(8, 12), 8, 12)
    assert e.value.code == 1 and "multiple of 64" in str(e.value)
