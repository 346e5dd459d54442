"""The C ABI without a GPU: the library loads and exports every symbol the
public headers declare, a device-less open fails with a message, and
exn_check_gguf applies open-dit's checks (src/weights.lisp:47-61)."""
import ctypes
import glob
import os
import re

import numpy as np
import pytest

import exn_b200 as E
from oracle import dit_oracle as O
from oracle.synth_gguf import write_gguf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TINY = dict(width=256, layers=2, ffn=768, context=256)


def declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"\b(exn_\w+)\s*\(", src))
    return sorted(names)


def test_headers_declare_the_boundary():
    d = declared()
    for name in ["exn_open", "exn_close", "exn_load_gguf", "exn_check_gguf", "exn_load_tensor",
                 "exn_velocity", "exn_generate", "exn_release", "exn_last_error"]:
        assert name in d


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(E.LIB_PATH)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert E.lib().exn_abi_version() == 1


def test_default_config_is_the_dit_shape():
    c = E.default_config()
    assert (c.width, c.layers, c.ffn, c.latent, c.context, c.freq, c.head_dim) == (4096, 32, 12288, 64, 4096, 256, 128)


def test_open_fails_cleanly_without_a_device():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(E.ExnError) as e:
        E.Dit(**TINY)
    assert e.value.code == 2 and "no CUDA device" in str(e.value)


def test_open_rejects_unsupported_shapes():
    with pytest.raises(E.ExnError) as e:
        E.Dit(width=300, layers=1, ffn=768, context=256)
    assert e.value.code == 1


@pytest.fixture(scope="module")
def tiny_sw():
    return O.SynthWeights.make(O.Shape(**TINY), seed=1)


def test_check_gguf_accepts_the_dit(tmp_path, tiny_sw):
    p = tmp_path / "dit.gguf"
    write_gguf(p, tiny_sw)
    E.check_gguf(p, **TINY)


@pytest.mark.parametrize("mtype", ["f32", "f16", "bf16"])
def test_check_gguf_accepts_unquantised_matrices(tmp_path, tiny_sw, mtype):
    p = tmp_path / "dit.gguf"
    write_gguf(p, tiny_sw, matrix_type=mtype)
    E.check_gguf(p, **TINY)


def test_check_gguf_lists_every_problem(tmp_path, tiny_sw):
    p = tmp_path / "bad.gguf"
    write_gguf(p, tiny_sw, arch="flux", drop=("proj_out.weight",), bad_dims="txt_in.out_layer.weight",
               extra=("transformer_blocks.9.attn.norm_q.weight", "stray.weight"))
    with pytest.raises(E.ExnError) as e:
        E.check_gguf(p, **TINY)
    msg = str(e.value)
    assert e.value.code == 3
    assert 'architecture "flux", not "qwen_image"' in msg
    assert "missing proj_out.weight" in msg
    assert "txt_in.out_layer.weight is (224 256), not (256 256)" in msg
    assert "1 tensors more than the model has" in msg


def test_check_gguf_wrong_shape_for_config(tmp_path, tiny_sw):
    p = tmp_path / "dit.gguf"
    write_gguf(p, tiny_sw)
    with pytest.raises(E.ExnError) as e:
        E.check_gguf(p, width=512, layers=2, ffn=768, context=256)
    assert "not (512 512)" in str(e.value)


def test_check_gguf_unreadable(tmp_path):
    with pytest.raises(E.ExnError) as e:
        E.check_gguf(tmp_path / "nope.gguf", **TINY)
    assert e.value.code == 5
    junk = tmp_path / "junk.gguf"
    junk.write_bytes(b"GGUF" + b"\x03\x00\x00\x00" + b"\xff" * 40)
    with pytest.raises(E.ExnError) as e:
        E.check_gguf(junk, **TINY)
    assert e.value.code == 5


def test_prefix_keys():
    assert E.prefix_key_of(None) == 0
    assert E.prefix_key_of("a prompt") == E.prefix_key_of("a prompt") != 0
    assert E.prefix_key_of(("edit", 1)) != E.prefix_key_of(("edit", 2))


def test_streaming_gguf_writer_equals_the_whole_file_writer(tmp_path):
    """The full-size upload test writes its 7.6 GB GGUF tensor by tensor; at a small shape that writer
    produces the same bytes as the writer the other tests use, and passes open-dit's checks."""
    from oracle.synth_gguf import write_gguf_streaming
    sh = O.Shape(**TINY)
    sw = O.SynthWeights.make(sh, seed=1)
    a, b = tmp_path / "a.gguf", tmp_path / "b.gguf"
    write_gguf(a, sw)
    write_gguf_streaming(b, sh, lambda name, dims: sw.vec[name] if len(dims) == 1 else sw.q8[name])
    assert a.read_bytes() == b.read_bytes()
    E.check_gguf(b, **TINY)
