"""The full-size GGUF upload (upload-dit, src/cuda-dit.lisp:52-86, which logs the gigabytes and
seconds of the load at :84-85): a 7.6 GB synthetic Q8_0 qwen_image GGUF of the D=4096, 32-block DiT
is written (tensor by tensor, the values from the library's synthetic generator, which the oracle's
generator reproduces bit for bit), checked and uploaded with exn_load_gguf, and the weights the
handle then holds are compared, by a digest of every byte, with exn_load_synthetic's."""
import os
import shutil
import time

import pytest

import exn_b200 as E
from oracle import dit_oracle as O
from oracle.synth_gguf import write_gguf_streaming
from test_gpu_full import DeviceWeights

pytestmark = pytest.mark.gpu


def test_full_gguf_upload_equals_synthetic(tmp_path):
    import ctypes
    if shutil.disk_usage(tmp_path).free < 12e9:
        pytest.skip("needs 12 GB of free disk for the 7.6 GB GGUF")
    sh = O.Shape()
    path = tmp_path / "dit_full.gguf"
    with E.Dit() as ref:
        ref.load_synthetic(1)
        want = ctypes.c_uint64()
        ref._ck(E.lib().exn_test_weights_digest(ref.h, ctypes.byref(want)))
        sw = DeviceWeights(ref, sh, seed=1)
        t0 = time.perf_counter()
        write_gguf_streaming(path, sh, lambda name, dims: sw(name) if len(dims) == 1 else sw.q8(name))
        t_write = time.perf_counter() - t0
    size = os.path.getsize(path)
    assert 7.5e9 < size < 7.7e9, size
    try:
        t0 = time.perf_counter()
        d = E.upload_dit(path)
        t_load = time.perf_counter() - t0
        got = ctypes.c_uint64()
        d._ck(E.lib().exn_test_weights_digest(d.h, ctypes.byref(got)))
        d.close()
    finally:
        os.remove(path)
    print("\nfull GGUF: %.2f GB written in %.1f s; exn_load_gguf (open-dit checks, upload, Q8_0 -> bf16 on the "
          "device) %.2f s = %.2f GB/s of file" % (size / 1e9, t_write, t_load, size / 1e9 / t_load))
    assert got.value == want.value
