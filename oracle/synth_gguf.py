"""Write a synthetic ``qwen_image`` DiT GGUF with gguf-py.  TEST INFRASTRUCTURE ONLY.

Used by tests/golden/make_golden.py (so the reference's own ``ref_dit.py``
reads the weights through its GGUFReader) and by the loader tests, which
also plant faults here, on the CPU: a wrong architecture, a missing or
extra tensor, a tensor with the wrong dims (the checks of open-dit,
src/weights.lisp:47-61).
"""
from __future__ import annotations

import numpy as np

from . import dit_oracle as O


def write_gguf(path, sw: "O.SynthWeights", arch="qwen_image", drop=(), extra=(), bad_dims=None,
               matrix_type="q8_0"):
    """MATRIX_TYPE: 'q8_0' (the weights as quantised), or 'f32' / 'f16' /
    'bf16' (the dequantised values in that type)."""
    import gguf
    wr = gguf.GGUFWriter(str(path), arch=arch)
    for name, dims in O.expected_tensors(sw.shape):
        if name in drop:
            continue
        full = O.PREFIX + name
        if len(dims) == 1:
            wr.add_tensor(full, sw.vec[name])
            continue
        qs, d = sw.q8[name]
        rows, cols = qs.shape
        if bad_dims and name == bad_dims:
            v = O.q8_0_dequantize(qs, d)[:, : cols - 32]
            wr.add_tensor(full, np.ascontiguousarray(v, dtype=np.float32))
        elif matrix_type == "q8_0":
            packed = O.q8_0_pack(qs, d).reshape(rows, cols // 32 * 34)
            wr.add_tensor(full, packed, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        elif matrix_type == "f32":
            wr.add_tensor(full, O.q8_0_dequantize(qs, d))
        elif matrix_type == "f16":
            wr.add_tensor(full, O.q8_0_dequantize(qs, d).astype(np.float16))
        elif matrix_type == "bf16":
            v = O.q8_0_dequantize(qs, d)
            bits = (v.view(np.uint32) + 0x7FFF + ((v.view(np.uint32) >> 16) & 1)) >> 16
            wr.add_tensor(full, bits.astype(np.uint16), raw_dtype=gguf.GGMLQuantizationType.BF16)
        else:
            raise ValueError(matrix_type)
    for name in extra:
        wr.add_tensor(O.PREFIX + name, np.zeros(32, dtype=np.float32))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()


def write_gguf_streaming(path, shape: "O.Shape", tensor, arch="qwen_image"):
    """A full-size synthetic GGUF written tensor by tensor, so only one tensor is in host memory at a
    time.  TENSOR(name, dims) gives a 1-D tensor as fp32, or a matrix as Q8_0 (qs int8 (rows, cols),
    d fp16 (rows, cols / 32))."""
    import gguf
    wr = gguf.GGUFWriter(str(path), arch=arch)
    specs = O.expected_tensors(shape)
    for name, dims in specs:
        if len(dims) == 1:
            wr.add_tensor_info(O.PREFIX + name, (dims[0],), np.dtype(np.float32), dims[0] * 4)
        else:
            cols, rows = dims
            wr.add_tensor_info(O.PREFIX + name, (rows, cols // 32 * 34), np.dtype(np.uint8), rows * cols // 32 * 34,
                               raw_dtype=gguf.GGMLQuantizationType.Q8_0)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_ti_data_to_file()
    for name, dims in specs:
        t = tensor(name, dims)
        if len(dims) == 1:
            wr.write_tensor_data(np.ascontiguousarray(t, dtype=np.float32))
        else:
            qs, d = t
            wr.write_tensor_data(O.q8_0_pack(qs, d).reshape(dims[1], dims[0] // 32 * 34))
    wr.close()
