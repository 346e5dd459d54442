"""CPU oracle for the prompt encoder (Qwen3-VL-8B's text model).  TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module; tests/ use it as the checker of the CUDA encoder
(exn_enc_states).  What it restates: ex-nihilo's ``encoder-states`` (src/encoder.lisp:143-183)
reads every token's state after the text model's LAST BLOCK, BEFORE its final norm, from illatio's
qwen3 forward, with the positions of ``mrope-table`` (src/encoder.lisp:26-39: Qwen3-VL's
interleaved M-RoPE, frequency j turning by h where j mod 3 is 1 and by w where it is 2, below 60,
by t elsewhere).  illatio is the sibling project the reference runs the encoder through and is
not in the reference tree; its qwen3 forward is the published Qwen3 architecture:

    x = embed[ids]
    per block:  h = rms(x) * attn_norm;  q, k, v = h Wq^T, h Wk^T, h Wv^T  (32 / 8 / 8 heads of 128)
                q, k = rms_head(q) * q_norm, rms_head(k) * k_norm;  RoPE on halves (j, j + 64)
                x += softmax_causal(q k^T / sqrt(128)) v  Wo^T      (query head i reads kv head i / 4)
                h = rms(x) * ffn_norm;  x += (silu(h Wg^T) * (h Wu^T)) Wd^T

Parity is pinned by tests/golden/make_encoder_golden.py, which loads this module's synthetic weights into
transformers' own ``Qwen3VLTextModel`` (fp32, eager attention) and stores the last block's output
for text positions and for an edit prompt's M-RoPE positions; tests/test_oracle.py holds this
module to it.

The synthetic weights come from the DiT's counter hash (oracle/dit_oracle.py ``synth_unit``):
tensor number i of ``encoder_tensors`` uses stream 30000 + i; matrices are N(0, std) quantised to
Q8_0 (as the reference's checkpoint stores them), vectors 1 + N(0, std) in fp32, so the CUDA
library makes the same bits (``exn_enc_load_synthetic``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import dit_oracle as D

STREAM0 = 30000


@dataclass(frozen=True)
class EncShape:
    """Qwen3-VL-8B's text model (the qwen3vl GGUF's metadata)."""
    width: int = 4096
    layers: int = 36
    heads: int = 32
    kv_heads: int = 8
    ffn: int = 12288
    vocab: int = 151936
    theta: float = 5000000.0
    eps: float = 1e-6
    head_dim: int = 128


SMALL = EncShape(width=512, layers=2, heads=4, kv_heads=2, ffn=1024, vocab=512)


def encoder_tensors(sh: EncShape):
    """(name, GGUF dims) of every tensor the encoder reads, dims innermost first as GGUF lists them
    (llama.cpp's qwen3vl names); the final norm and the LM head are not read."""
    w, q, kv = sh.width, sh.heads * sh.head_dim, sh.kv_heads * sh.head_dim
    r = [("token_embd.weight", (w, sh.vocab))]
    for i in range(sh.layers):
        b = "blk.%d." % i
        r += [(b + "attn_norm.weight", (w,)), (b + "attn_q.weight", (w, q)), (b + "attn_k.weight", (w, kv)),
              (b + "attn_v.weight", (w, kv)), (b + "attn_q_norm.weight", (sh.head_dim,)),
              (b + "attn_k_norm.weight", (sh.head_dim,)), (b + "attn_output.weight", (q, w)),
              (b + "ffn_norm.weight", (w,)), (b + "ffn_gate.weight", (w, sh.ffn)), (b + "ffn_up.weight", (w, sh.ffn)),
              (b + "ffn_down.weight", (sh.ffn, w))]
    return r


def synth_std(sh: EncShape) -> float:
    return D.synth_std(sh.width)


@dataclass
class SynthEncoder:
    """The encoder's synthetic weights: matrices as Q8_0 (qs, d), vectors fp32, made on first use."""
    shape: EncShape
    seed: int = 1
    index: dict = field(default_factory=dict)
    cache: dict = field(default_factory=dict)

    def __post_init__(self):
        self.index = {n: (i, d) for i, (n, d) in enumerate(encoder_tensors(self.shape))}

    def q8(self, name):
        """(qs int8 (rows, cols), d fp16 (rows, cols / 32)) of a matrix."""
        i, dims = self.index[name]
        v = D.synth_normal(self.seed, STREAM0 + i, tuple(reversed(dims)), synth_std(self.shape))
        return D.q8_0_quantize(v)

    def __call__(self, name):
        if name not in self.cache:
            i, dims = self.index[name]
            if len(dims) == 1:
                v = np.float32(1.0) + D.synth_normal(self.seed, STREAM0 + i, dims, synth_std(self.shape))
                self.cache[name] = v.astype(np.float32)
            else:
                self.cache[name] = D.q8_0_dequantize(*self.q8(name))
        return self.cache[name]


def synth_ids(sh: EncShape, n: int, seed: int = 0) -> np.ndarray:
    """N token ids in [0, vocab) from the counter hash (stream 3100)."""
    return (D.synth_unit(seed, 3100, n).astype(np.int64) % sh.vocab).astype(np.int32)


def text_positions(n: int) -> np.ndarray:
    """A text prompt's positions: (i, i, i) for token i (src/encoder.lisp:118, plain prompts)."""
    return np.repeat(np.arange(n, dtype=np.int32)[:, None], 3, axis=1)


def edit_positions(a0: int, gh: int, gw: int, tail: int) -> np.ndarray:
    """An edit prompt's positions (src/encoder.lisp:119-123): A0 text tokens at (i, i, i), the
    picture's GH x GW pads at (a0, a0 + r, a0 + c), then TAIL text tokens from a0 + max(gh, gw)."""
    pos = [(i, i, i) for i in range(a0)]
    pos += [(a0, a0 + r, a0 + c) for r in range(gh) for c in range(gw)]
    p0 = a0 + max(gh, gw)
    pos += [(p0 + i, p0 + i, p0 + i) for i in range(tail)]
    return np.asarray(pos, dtype=np.int32)


def mrope_angles(sh: EncShape, positions: np.ndarray) -> np.ndarray:
    """(n, 64) rotation angles: frequency j of theta^(-2j/128) turned by the t, h or w position of
    mrope-table's rule (src/encoder.lisp:26-39), in float64."""
    half = sh.head_dim // 2
    j = np.arange(half)
    inv = sh.theta ** (-(2.0 * j) / sh.head_dim)
    axis = np.where(j < 60, j % 3, 0)
    pos = positions.astype(np.float64)[:, axis]                  # (n, 64)
    return pos * inv[None, :]


def rms(x, w, eps):
    x = x.astype(np.float32)
    return (x / np.sqrt((x * x).mean(-1, keepdims=True) + np.float32(eps))) * w


def rope_halves(x, cos, sin):
    """x (n, heads, 128): pairs (j, j + 64) rotated by angle j (Qwen3's rotate_half form)."""
    a, b = x[..., :64], x[..., 64:]
    c, s = cos[:, None, :], sin[:, None, :]
    return np.concatenate([a * c - b * s, a * s + b * c], axis=-1)


def attention_causal(q, k, v, group):
    """q (n, H, 128), k / v (n, KV, 128); query head i reads kv head i // group; causal."""
    n, nh, hd = q.shape
    out = np.empty_like(q)
    mask = np.triu(np.ones((n, n), dtype=bool), 1)
    for h in range(nh):
        kh, vh = k[:, h // group], v[:, h // group]
        s = (q[:, h].astype(np.float64) @ kh.T.astype(np.float64)) / math.sqrt(hd)
        s[mask] = -np.inf
        s = np.exp(s - s.max(-1, keepdims=True))
        out[:, h] = ((s / s.sum(-1, keepdims=True)) @ vh.astype(np.float64)).astype(np.float32)
    return out


def block(wt, sh: EncShape, i: int, x, cos, sin):
    b = "blk.%d." % i
    n = x.shape[0]
    h = rms(x, wt(b + "attn_norm.weight"), sh.eps)
    q = (h @ wt(b + "attn_q.weight").T).reshape(n, sh.heads, sh.head_dim)
    k = (h @ wt(b + "attn_k.weight").T).reshape(n, sh.kv_heads, sh.head_dim)
    v = (h @ wt(b + "attn_v.weight").T).reshape(n, sh.kv_heads, sh.head_dim)
    q = rope_halves(rms(q, wt(b + "attn_q_norm.weight"), sh.eps), cos, sin)
    k = rope_halves(rms(k, wt(b + "attn_k_norm.weight"), sh.eps), cos, sin)
    a = attention_causal(q, k, v, sh.heads // sh.kv_heads).reshape(n, -1)
    x = x + a @ wt(b + "attn_output.weight").T
    h = rms(x, wt(b + "ffn_norm.weight"), sh.eps)
    g = h @ wt(b + "ffn_gate.weight").T
    u = h @ wt(b + "ffn_up.weight").T
    return (x + ((g / (1 + np.exp(-g))) * u) @ wt(b + "ffn_down.weight").T).astype(np.float32)


def states(wt, sh: EncShape, ids, positions=None, layers=None):
    """encoder-states: every token's state after the last block (or after LAYERS blocks), before
    the final norm: (n, width) float32."""
    ids = np.asarray(ids)
    pos = text_positions(len(ids)) if positions is None else np.asarray(positions)
    ang = mrope_angles(sh, pos)
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    x = wt("token_embd.weight")[ids].astype(np.float32)
    for i in range(sh.layers if layers is None else layers):
        x = block(wt, sh, i, x, cos, sin)
    return x


def write_gguf(path, wt: SynthEncoder, arch="qwen3vl", matrix_type="q8_0", drop=(), extra=(), bad_dims=None):
    """The synthetic encoder as a GGUF with gguf-py, llama.cpp's tensor names.  MATRIX_TYPE 'q8_0'
    (the quantised values), 'bf16' or 'f32' (the dequantised ones); the embedding table goes the
    same way.  DROP / EXTRA / BAD_DIMS plant the faults the loader must name (on the CPU)."""
    import gguf
    wr = gguf.GGUFWriter(str(path), arch=arch)
    for name, dims in encoder_tensors(wt.shape):
        if name in drop:
            continue
        if len(dims) == 1:
            wr.add_tensor(name, wt(name))
            continue
        qs, d = wt.q8(name)
        rows, cols = qs.shape
        if bad_dims == name:
            wr.add_tensor(name, np.ascontiguousarray(D.q8_0_dequantize(qs, d)[:, : cols - 32]))
        elif matrix_type == "q8_0":
            wr.add_tensor(name, D.q8_0_pack(qs, d).reshape(rows, cols // 32 * 34),
                          raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        elif matrix_type == "f32":
            wr.add_tensor(name, D.q8_0_dequantize(qs, d))
        elif matrix_type == "bf16":
            v = D.q8_0_dequantize(qs, d)
            u = v.view(np.uint32)
            bits = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
            wr.add_tensor(name, bits.astype(np.uint16), raw_dtype=gguf.GGMLQuantizationType.BF16)
        else:
            raise ValueError(matrix_type)
    for name in extra:
        wr.add_tensor(name, np.ones(wt.shape.width, dtype=np.float32))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
