"""CPU oracle for the VAE decoder (the step after the DiT).  TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module; tests/ use it as the checker of the CUDA decoder
(exn_vae_decode).  It restates the reference's numpy decoder, ``inspect/ref_vae.py`` of ex-nihilo
(conv :31-44, rms :47-49, silu :52-53, resblock :56-62, attention :65-74, dupup :77-83, decode
:86-104), with the weights given by a callable instead of a safetensors file, and the schema of
``src/weights.lisp:63-100`` (``+vae-stages+``, ``vae-expected``).

Parity is pinned by tests/golden/make_golden.py, which writes this module's synthetic weights as a
real safetensors file, runs the reference's own ``ref_vae.decode`` on it and stores the picture;
tests/test_oracle.py holds this module to that picture.

The synthetic weights come from the same counter hash as the DiT's (oracle/dit_oracle.py
``synth_unit``), streams 20000 + the tensor's index in ``vae_expected``, every value rounded to
bf16 (a checkpoint's type), so the CUDA library makes the same bits (``exn_vae_load_synthetic``).
"""
from __future__ import annotations

import math

import numpy as np

from . import dit_oracle as D

# (in, out, spatial up, temporal up), deepest first: src/weights.lisp:63-65, ref_vae.py:15-16
STAGES = ((1152, 1152, True, True), (1152, 1152, True, True), (1152, 576, True, True), (576, 288, True, False),
          (288, 144, False, False))
Z, OUT = 64, 4


def vae_expected(stages=STAGES, z=Z, out=OUT):
    """(name, shape) of every decoder tensor, shapes row-major, in vae-expected's order
    (src/weights.lisp:67-100)."""
    r = []

    def conv(name, o, i, k, frames=True):
        r.append((name + ".weight", (o, i, 1, k, k) if frames else (o, i, k, k)))
        r.append((name + ".bias", (o,)))

    def res(p, i, o):
        r.append((p + ".residual.0.gamma", (i, 1, 1, 1)))
        conv(p + ".residual.2", o, i, 3)
        r.append((p + ".residual.3.gamma", (o, 1, 1, 1)))
        conv(p + ".residual.6", o, o, 3)
        if i != o:
            conv(p + ".shortcut", o, i, 1)

    top = stages[0][0]
    conv("conv2", z, z, 1)
    conv("decoder.conv1", top, z, 3)
    res("decoder.middle.0", top, top)
    r.append(("decoder.middle.1.norm.gamma", (top, 1, 1)))
    conv("decoder.middle.1.to_qkv", 3 * top, top, 1, frames=False)
    conv("decoder.middle.1.proj", top, top, 1, frames=False)
    res("decoder.middle.2", top, top)
    for s, (i, o, up, tup) in enumerate(stages):
        for j in range(3):
            res("decoder.upsamples.%d.upsamples.%d" % (s, j), i if j == 0 else o, o)
        if up:
            conv("decoder.upsamples.%d.upsamples.3.resample.1" % s, o, o, 3, frames=False)
            if tup:
                conv("decoder.upsamples.%d.upsamples.3.time_conv" % s, 2 * o, o, 1)
    r.append(("decoder.head.0.gamma", (stages[-1][1], 1, 1, 1)))
    conv("decoder.head.2", out, stages[-1][1], 3)
    return r


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even), kept as fp32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


class SynthVae:
    """The decoder's synthetic weights: weight N(0, 1/fan_in), bias N(0, 0.02), gamma 1 + N(0, 0.1),
    each rounded to bf16.  Made on first use of each tensor."""

    def __init__(self, seed=1):
        self.seed = seed
        self.spec = vae_expected()
        self.index = {n: (i, s) for i, (n, s) in enumerate(self.spec)}
        self.cache = {}

    def __call__(self, name):
        if name not in self.cache:
            i, shape = self.index[name]
            leaf = name.rsplit(".", 1)[1]
            std, base = 0.02, 0.0
            if leaf == "weight":
                std = 1.0 / math.sqrt(float(np.prod(shape[1:])))
            elif leaf == "gamma":
                std, base = 0.1, 1.0
            n = int(np.prod(shape))
            v = D.synth_unit(self.seed, 20000 + i, n).astype(np.float32) * np.float32(std / D._IH_STD)
            if base:
                v = np.float32(base) + v
            self.cache[name] = bf16_round(v).reshape(shape)
        return self.cache[name]


# ---------------------------------------------------------------------------- ref_vae.py's decoder

def conv(x, w, b, k):
    """x: C x H x W; w: O x C x [1 x] k x k; 'same' padding, stride 1 (ref_vae.py:31-44)."""
    w = w.reshape(w.shape[0], w.shape[1], k, k)
    c, h, wd = x.shape
    if k == 1:
        return (w[:, :, 0, 0] @ x.reshape(c, -1)).reshape(-1, h, wd) + b[:, None, None]
    xp = np.pad(x, ((0, 0), (1, 1), (1, 1)))
    out = np.zeros((w.shape[0], h * wd), dtype=np.float32)
    for dy in range(3):
        for dx in range(3):
            out += w[:, :, dy, dx] @ xp[:, dy:dy + h, dx:dx + wd].reshape(c, -1)
    return out.reshape(-1, h, wd) + b[:, None, None]


def rms(x, gamma):                               # ref_vae.py:47-49
    n = np.sqrt((x * x).sum(0, keepdims=True))
    return x / np.maximum(n, 1e-12) * np.sqrt(x.shape[0]) * gamma.reshape(-1, 1, 1)


def silu(x):                                     # ref_vae.py:52-53
    return x / (1 + np.exp(-x))


def resblock(wt, p, x):                          # ref_vae.py:56-62
    i = x.shape[0]
    o = wt(p + ".residual.2.weight").shape[0]
    h = conv(x, wt(p + ".shortcut.weight"), wt(p + ".shortcut.bias"), 1) if i != o else x
    y = conv(silu(rms(x, wt(p + ".residual.0.gamma"))), wt(p + ".residual.2.weight"), wt(p + ".residual.2.bias"), 3)
    y = conv(silu(rms(y, wt(p + ".residual.3.gamma"))), wt(p + ".residual.6.weight"), wt(p + ".residual.6.bias"), 3)
    return (y + h).astype(np.float32)


def attention(wt, p, x):                         # ref_vae.py:65-74
    c, h, w = x.shape
    y = rms(x, wt(p + ".norm.gamma"))
    qkv = conv(y, wt(p + ".to_qkv.weight"), wt(p + ".to_qkv.bias"), 1).reshape(3 * c, h * w).T
    q, k, v = qkv[:, :c], qkv[:, c:2 * c], qkv[:, 2 * c:]
    s = q @ k.T / np.sqrt(c)
    s = np.exp(s - s.max(-1, keepdims=True))
    a = (s / s.sum(-1, keepdims=True)) @ v
    return (conv(a.T.reshape(c, h, w), wt(p + ".proj.weight"), wt(p + ".proj.bias"), 1) + x).astype(np.float32)


def dupup(x, out_c, ft, fs=2):                   # ref_vae.py:77-83
    c, h, w = x.shape
    rep = out_c * ft * fs * fs // c
    x = np.repeat(x, rep, axis=0).reshape(out_c, ft, fs, fs, h, w)[:, ft - 1]
    return x.transpose(0, 3, 1, 4, 2).reshape(out_c, h * fs, w * fs)


def decode(wt, z, trace=None):
    """z: 64 x H x W (denormalised) -> 4 x 16H x 16W in -1 .. 1 (ref_vae.py:86-104).  TRACE, a list,
    receives the stream after the middle and after each stage (C x H x W)."""
    x = conv(z, wt("conv2.weight"), wt("conv2.bias"), 1)
    x = conv(x, wt("decoder.conv1.weight"), wt("decoder.conv1.bias"), 3)
    x = resblock(wt, "decoder.middle.0", x)
    x = attention(wt, "decoder.middle.1", x)
    x = resblock(wt, "decoder.middle.2", x)
    if trace is not None:
        trace.append(x)
    for s, (i, o, up, tup) in enumerate(STAGES):
        x0 = x
        for j in range(3):
            x = resblock(wt, "decoder.upsamples.%d.upsamples.%d" % (s, j), x)
        if up:
            x = np.repeat(np.repeat(x, 2, axis=1), 2, axis=2)
            p = "decoder.upsamples.%d.upsamples.3.resample.1" % s
            x = conv(x, wt(p + ".weight"), wt(p + ".bias"), 3)
            x = x + dupup(x0, o, 2 if tup else 1)
        if trace is not None:
            trace.append(x)
    x = silu(rms(x, wt("decoder.head.0.gamma")))
    x = conv(x, wt("decoder.head.2.weight"), wt("decoder.head.2.bias"), 3)
    return np.clip(x, -1, 1).astype(np.float32)


def write_safetensors(path, tensors):
    """TENSORS: [(name, fp32 array already bf16-representable)] -> a BF16 safetensors file."""
    import json
    import struct
    header, blobs, off = {}, [], 0
    for name, a in tensors:
        raw = (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> np.uint32(16)).astype(np.uint16).tobytes()
        header[name] = {"dtype": "BF16", "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
