"""CPU oracle for the Qwen-Image-2.1 DiT hot path.  TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this module.  Only tests/, the smoke check in
__graft_entry__.py and the CPU legs of bench.py (``cpu_baseline`` and
``--impl reference``) may use it, and only as the checker or as the timed CPU
baseline, never as the thing the GPU path computes with.

What it restates (paths relative to the ex-nihilo project):

* the fp32 numpy DiT of ``inspect/ref_dit.py`` (its ``forward``, lines
  108-153, and helpers 33-105), generalised to a runtime shape (width, FFN,
  layers, context width) so small cases run in seconds;
* the edit layout that ``ref_dit.py`` lacks: positions from
  ``src/host.lisp:37-50`` (``dit-positions``) and the mask from
  ``src/cuda/dit.cu:60-66`` (``xa_lim``);
* the step loop of ``src/generate.lisp:133-135`` (Euler, fixed Turbo sigmas of
  ``src/generate.lisp:7-9``);
* Q8_0 (32 int8 + an fp16 scale per block) exactly as gguf-py 0.19.0's
  ``Q8_0.quantize_blocks`` / ``dequantize_blocks`` compute it (gguf-py is the
  third-party package ``ref_dit.py`` imports; it is not vendored in the
  reference tree);
* the tensor schema of ``src/weights.lisp:19-45`` (``dit-shape``,
  ``dit-expected``).

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
``inspect/ref_dit.py`` (imported, its module constants patched to the shape)
on weights and inputs from this module's generator and stores the outputs in
``tests/golden/``; ``tests/test_oracle.py`` holds this module to them.

The synthetic weight/input generator (``synth_*``) is this build's own: a
counter-based hash so the CUDA library can produce bit-identical Q8_0 weights
on the device (``exn_load_synthetic``) without shipping gigabytes.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

PREFIX = "model.diffusion_model."
TURBO_SIGMAS = (1.0, 0.978453, 0.95418, 0.926626, 0.89508, 0.845148, 0.704534, 0.414568, 0.0)
ROPE_AXES = (16, 56, 56)          # ref_dit.py:20, host.lisp:17
HEAD_DIM = 128                    # ref_dit.py:19
LN_EPS = 1e-6                     # ref_dit.py:37, 43

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30


@dataclass(frozen=True)
class Shape:
    """``dit-shape`` of src/weights.lisp:19-20, with the block count and
    width free so the small parity cases run in seconds."""
    width: int = 4096
    layers: int = 32
    ffn: int = 12288
    latent: int = 64
    context: int = 4096
    freq: int = 256
    head_dim: int = HEAD_DIM

    @property
    def heads(self) -> int:
        return self.width // self.head_dim


def expected_tensors(sh: Shape):
    """(name, dims) of every DiT tensor, dims in ggml order (contiguous axis
    first), in the order of ``dit-expected`` (src/weights.lisp:22-45)."""
    w, f = sh.width, sh.ffn
    out = [("img_in.weight", (sh.latent, w)),
           ("txt_in.text_norm.weight", (sh.context,)),
           ("txt_in.in_layer.weight", (sh.context, w)),
           ("txt_in.out_layer.weight", (w, w)),
           ("time_text_embed.timestep_embedder.linear_1.weight", (sh.freq, w)),
           ("time_text_embed.timestep_embedder.linear_2.weight", (w, w)),
           ("modulation.1.weight", (w, 4 * w)),
           ("norm_out.linear.weight", (w, w)),
           ("proj_out.weight", (w, sh.latent))]
    for i in range(sh.layers):
        b = "transformer_blocks.%d." % i
        out += [(b + "attn.norm_q.weight", (sh.head_dim,)),
                (b + "attn.norm_k.weight", (sh.head_dim,)),
                (b + "attn.to_q.weight", (w, w)),
                (b + "attn.to_k.weight", (w, w)),
                (b + "attn.to_v.weight", (w, w)),
                (b + "attn.to_out.0.weight", (w, w)),
                (b + "img_mlp.gate_up.weight", (w, 2 * f)),
                (b + "img_mlp.out.weight", (f, w))]
    return out


# --------------------------------------------------------------------------- Q8_0

def q8_0_quantize(x: np.ndarray):
    """fp32 values (last axis a multiple of 32) -> (qs int8 [..., n], d fp16
    [..., n/32]).  The arithmetic of gguf-py 0.19.0 ``Q8_0.quantize_blocks``:
    d = max|x| / 127 in fp32, q = round-half-away(x * (1/d)), d stored fp16."""
    x = np.asarray(x, dtype=np.float32)
    blocks = x.reshape(-1, 32)
    d = np.abs(blocks).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    y = blocks * inv
    a = np.abs(y)
    fl = np.floor(a)
    q = np.sign(y) * (fl + np.floor(np.float32(2) * (a - fl)))
    qs = q.astype(np.int8).reshape(x.shape)
    dd = d.astype(np.float16).reshape(x.shape[:-1] + (x.shape[-1] // 32,))
    return qs, dd


def q8_0_dequantize(qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    """int8 q times its block's fp16 scale, in fp32 (gguf-py
    ``Q8_0.dequantize_blocks``)."""
    n = qs.shape[-1]
    w = qs.reshape(-1, n // 32, 32).astype(np.float32) * d.reshape(-1, n // 32, 1).astype(np.float32)
    return w.reshape(qs.shape)


def q8_0_pack(qs: np.ndarray, d: np.ndarray) -> np.ndarray:
    """GGUF's 34-byte Q8_0 blocks: fp16 d then 32 int8."""
    nb = qs.size // 32
    out = np.empty((nb, 34), dtype=np.uint8)
    out[:, :2] = d.reshape(nb, 1).view(np.uint8)
    out[:, 2:] = qs.reshape(nb, 32).view(np.uint8)
    return out.reshape(-1)


# --------------------------------------------------------------------------- synthetic data

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
_GOLD = np.uint64(0x9E3779B97F4A7C15)
# std of the sum of four independent uniform 16-bit integers
_IH_STD = math.sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0)
_IH_MEAN = 4 * 65535 // 2  # 131070


def _mix64(x: np.ndarray) -> np.ndarray:
    """splitmix64's finaliser (public-domain mixing function)."""
    x = x.astype(np.uint64)
    with np.errstate(over="ignore"):
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        x = x ^ (x >> np.uint64(31))
    return x


def synth_unit(seed: int, stream: int, count: int, start: int = 0) -> np.ndarray:
    """Approximately N(0,1) integers-derived floats: counter (stream << 32 |
    index) hashed by splitmix64, its four 16-bit fields summed (Irwin-Hall, 4
    terms) and centred.  Returned as the exact integer offsets (int32); the
    float value is ``offset * scale`` with ``scale`` a float32 constant, so the
    CUDA generator reproduces every bit."""
    chunk = 1 << 20
    if count > chunk:  # in cache-sized pieces: the same values, twice as fast for large tensors
        out = np.empty(count, dtype=np.int32)
        for s in range(0, count, chunk):
            out[s:s + min(chunk, count - s)] = synth_unit(seed, stream, min(chunk, count - s), start + s)
        return out
    idx = np.arange(start, start + count, dtype=np.uint64)
    with np.errstate(over="ignore"):
        c = (np.uint64(stream) << np.uint64(32)) | idx
        h = _mix64(c + np.uint64(seed) * _GOLD)
    m = np.uint64(0xFFFF)
    s = (h & m) + ((h >> np.uint64(16)) & m) + ((h >> np.uint64(32)) & m) + (h >> np.uint64(48))
    return s.astype(np.int64).astype(np.int32) - np.int32(_IH_MEAN)


def synth_scale(std: float) -> np.float32:
    return np.float32(std / _IH_STD)


def synth_normal(seed: int, stream: int, shape, std: float = 1.0) -> np.ndarray:
    n = int(np.prod(shape))
    return (synth_unit(seed, stream, n).astype(np.float32) * synth_scale(std)).reshape(shape)


def synth_std(width: int) -> float:
    """0.02 at the model's width 4096, scaled by sqrt(4096 / width) so a
    narrow test DiT's activations and gates have the full model's statistics."""
    return 0.02 * math.sqrt(4096.0 / width)


def synth_tensor_f32(seed: int, index: int, name: str, dims, std: float) -> np.ndarray:
    """The fp32 value of synthetic tensor number INDEX (its position in
    ``expected_tensors``).  Matrices N(0, std); norm weights 1 + N(0, std);
    ``txt_in.text_norm.weight`` N(0, std) (it is used as 1 + w, ref_dit.py:120)."""
    shape = tuple(reversed(dims))                    # numpy (rows, cols)
    v = synth_normal(seed, index, shape, std)
    if len(dims) == 1 and not name.endswith("text_norm.weight"):
        v = np.float32(1.0) + v
    return v.astype(np.float32)


@dataclass
class SynthWeights:
    """Every tensor of a synthetic DiT: 2-D ones as Q8_0 (qs, d), 1-D ones
    as fp32, exactly as the CUDA library's ``exn_load_synthetic`` makes them."""
    shape: Shape
    seed: int = 1
    q8: dict = field(default_factory=dict)     # name -> (qs int8 (rows, cols), d fp16 (rows, cols/32))
    vec: dict = field(default_factory=dict)    # name -> fp32 (n,)

    @classmethod
    def make(cls, shape: Shape, seed: int = 1, only=None):
        """ONLY, a predicate on tensor names, restricts the set made (each
        tensor's values depend on its index in the full list, not on the set)."""
        sw = cls(shape, seed)
        std = synth_std(shape.width)
        for i, (name, dims) in enumerate(expected_tensors(shape)):
            if only is not None and not only(name):
                continue
            v = synth_tensor_f32(seed, i, name, dims, std)
            if len(dims) == 1:
                sw.vec[name] = v
            else:
                sw.q8[name] = q8_0_quantize(v)
        return sw

    def __call__(self, name: str) -> np.ndarray:
        """fp32 weight as gguf-py's dequantisation gives it (ref_dit.py:28-30)."""
        if name in self.vec:
            return self.vec[name]
        qs, d = self.q8[name]
        return q8_0_dequantize(qs, d)


def synth_inputs(sh: Shape, p: int, h: int, w: int, seed: int = 0, batch: int = 1):
    """Context (batch, P, context) and noise latent (batch, 64, H, W), ~N(0,1),
    from the same counter hash (streams 1000 + 2b, 1001 + 2b)."""
    ctx = np.stack([synth_normal(seed, 1000 + 2 * b, (p, sh.context)) for b in range(batch)])
    lat = np.stack([synth_normal(seed, 1001 + 2 * b, (sh.latent, h, w)) for b in range(batch)])
    return ctx.astype(np.float32), lat.astype(np.float32)


# --------------------------------------------------------------------------- the DiT's pieces

def linear(x, w):                       # ref_dit.py:33-34; w is (out, in)
    return x @ w.T


def layernorm(x, eps=LN_EPS):           # ref_dit.py:37-40
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    return (x - m) / np.sqrt(v + eps)


def rmsnorm(x, w, eps=LN_EPS):          # ref_dit.py:43-44
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w


def gelu_tanh(x):                       # ref_dit.py:47-48
    return 0.5 * x * (1 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def silu(x):                            # ref_dit.py:51-52
    return x / (1 + np.exp(-x))


def timestep_embedding(t, dim=256, period=10000.0):
    """cos half then sin half (ref_dit.py:55-59, host.lisp:9-15)."""
    half = dim // 2
    f = np.exp(-math.log(period) * np.arange(half, dtype=np.float32) / half)
    a = t * f
    return np.concatenate([np.cos(a), np.sin(a)]).astype(np.float32)


def image_positions(frame, h, w):
    """host.lisp:32-35: (frame, row, col), rows and columns centred on 0."""
    return [(frame, r - (h - h // 2), c - (w - w // 2)) for r in range(h) for c in range(w)]


def dit_positions(p, h, w, ref=None):
    """Every row's (frame, row, col), host.lisp:37-50.  P counts the whole
    prefix (text and reference picture).  REF = (A, RH, RW): A text rows,
    the RH x RW reference picture at frame A, the remaining text going on from
    A + max(RH, RW), the target picture after it."""
    if ref is None:
        return [(i, i, i) for i in range(p)] + image_positions(p, h, w)
    a, rh, rw = ref
    after = p - a - rh * rw
    pos = a + max(rh, rw)
    return ([(i, i, i) for i in range(a)] + image_positions(a, rh, rw)
            + [(pos + i,) * 3 for i in range(after)] + image_positions(pos + after, h, w))


def rope_tables(pos, theta=10000.0):
    """cos, sin: tokens x 64 (ref_dit.py:72-79)."""
    pos = np.asarray(pos, dtype=np.float32)
    angs = []
    for a, d in enumerate(ROPE_AXES):
        omega = 1.0 / theta ** (np.arange(0, d, 2, dtype=np.float64) / d)
        angs.append(pos[:, a:a + 1].astype(np.float64) * omega[None, :])
    ang = np.concatenate(angs, axis=1)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rope(x, cos, sin):                  # ref_dit.py:82-88; x tokens x heads x 128
    x0, x1 = x[..., 0::2], x[..., 1::2]
    c, s = cos[:, None, :], sin[:, None, :]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out


def xa_lim(g, p, l, b0, b1):
    """Last key row G sees (src/cuda/dit.cu:64-66): image rows all L keys, a
    reference picture's rows B0..B1-1 their block whole, other prefix rows
    causal.  Works on numpy arrays of G."""
    g = np.asarray(g)
    return np.where(g >= p, l - 1, np.where((g >= b0) & (g < b1), b1 - 1, g))


def attention(q, k, v, q0, p, l, b0=0, b1=0):
    """Masked softmax attention (ref_dit.py:91-105 with dit.cu's mask): Q rows
    are sequence rows Q0.., K/V have L rows; scale 1/sqrt(128)."""
    n, heads, hd = q.shape
    out = np.empty_like(q)
    scale = 1.0 / math.sqrt(hd)
    lim = xa_lim(np.arange(q0, q0 + n), p, l, b0, b1)
    mask = np.arange(l)[None, :] > lim[:, None]
    for h in range(heads):
        s = (q[:, h, :] @ k[:, h, :].T) * scale
        s = np.where(mask, -np.inf, s)
        s = s - s.max(-1, keepdims=True)
        e = np.exp(s)
        out[:, h, :] = (e / e.sum(-1, keepdims=True)) @ v[:, h, :]
    return out


def modulation(wt, sh: Shape, sigma):
    """The shared modulation rows (ref_dit.py:112-118) and norm_out's scale
    (ref_dit.py:150): (emb, [scale1, gate1, scale2, gate2] each 2 x W, sc 1 x W)."""
    W = sh.width
    t = sigma * 1000.0
    emb = np.stack([timestep_embedding(t, sh.freq), timestep_embedding(0.0, sh.freq)])
    emb = linear(silu(linear(emb, wt("time_text_embed.timestep_embedder.linear_1.weight"))),
                 wt("time_text_embed.timestep_embedder.linear_2.weight"))
    emb = silu(emb)
    mod = linear(emb, wt("modulation.1.weight"))
    pieces = [mod[:, i * W:(i + 1) * W] for i in range(4)]
    sc = linear(emb[0:1], wt("norm_out.linear.weight"))
    return emb, pieces, sc


def block(wt, sh: Shape, il, x, pieces, row, cos, sin, p, b0=0, b1=0):
    """Block IL on the sequence X (ref_dit.py:133-146): PIECES = the
    modulation rows (scale1, gate1, scale2, gate2), ROW the modulation row of
    each sequence row (0 image, 1 prefix), COS/SIN its RoPE tables."""
    W, HD, heads = sh.width, sh.head_dim, sh.heads
    scale1, gate1, scale2, gate2 = pieces
    n = x.shape[0]
    b = "transformer_blocks.%d." % il
    y = layernorm(x) * (1.0 + scale1[row])
    q = linear(y, wt(b + "attn.to_q.weight")).reshape(n, heads, HD)
    k = linear(y, wt(b + "attn.to_k.weight")).reshape(n, heads, HD)
    v = linear(y, wt(b + "attn.to_v.weight")).reshape(n, heads, HD)
    q = rope(rmsnorm(q, wt(b + "attn.norm_q.weight")), cos, sin)
    k = rope(rmsnorm(k, wt(b + "attn.norm_k.weight")), cos, sin)
    att = attention(q, k, v, 0, p, n, b0, b1).reshape(n, W)
    x = x + np.tanh(gate1[row]) * linear(att, wt(b + "attn.to_out.0.weight"))
    y = layernorm(x) * (1.0 + scale2[row])
    gu = linear(y, wt(b + "img_mlp.gate_up.weight"))
    y = silu(gu[:, :sh.ffn]) * gu[:, sh.ffn:]
    x = x + np.tanh(gate2[row]) * linear(y, wt(b + "img_mlp.out.weight"))
    return x.astype(np.float32)


def forward(wt, sh: Shape, ctx, latent, sigma, ref=None, trace=None):
    """The velocity (64 x H x W) at SIGMA: ref_dit.py:108-153, with the edit
    reference of src/cuda-dit.lisp:137-192 when REF = (A, ref_latent 64 x RH x
    RW): the reference picture's rows go into the prefix after text row A.
    TRACE, a list, receives txt_in's output and x after every block."""
    ptext = ctx.shape[0]
    c, h, w = latent.shape
    _, (scale1, gate1, scale2, gate2), sc = modulation(wt, sh, sigma)
    txt = rmsnorm(ctx, 1.0 + wt("txt_in.text_norm.weight"))
    txt = linear(gelu_tanh(linear(txt, wt("txt_in.in_layer.weight"))), wt("txt_in.out_layer.weight"))
    img = linear(latent.reshape(c, h * w).T, wt("img_in.weight"))
    if trace is not None:
        trace.append(txt.astype(np.float32))
    if ref is None:
        x = np.concatenate([txt, img]).astype(np.float32)
        p, b0, b1, refpos = ptext, 0, 0, None
    else:
        a, rlat = ref
        rc, rh, rw = rlat.shape
        rimg = linear(rlat.reshape(rc, rh * rw).T, wt("img_in.weight"))
        x = np.concatenate([txt[:a], rimg, txt[a:], img]).astype(np.float32)
        p, b0, b1, refpos = ptext + rh * rw, a, a + rh * rw, (a, rh, rw)
    n = x.shape[0]
    row = np.where(np.arange(n) < p, 1, 0)
    cos, sin = rope_tables(dit_positions(p, h, w, refpos))
    for il in range(sh.layers):
        x = block(wt, sh, il, x, (scale1, gate1, scale2, gate2), row, cos, sin, p, b0, b1)
        if trace is not None:
            trace.append(x)
    x = x[p:]
    x = layernorm(x) * (1.0 + sc)
    v = linear(x, wt("proj_out.weight"))
    return v.T.reshape(c, h, w).astype(np.float32)


def euler(wt, sh: Shape, ctx, z, sigmas=TURBO_SIGMAS, ref=None, velocities=None):
    """src/generate.lisp:133-135: z += (s' - s) * v for each pair of sigmas,
    the difference taken in double and rounded to single as the Lisp does."""
    z = np.array(z, dtype=np.float32, copy=True)
    for s, s2 in zip(sigmas[:-1], sigmas[1:]):
        v = forward(wt, sh, ctx, z, s, ref=ref)
        if velocities is not None:
            velocities.append(v)
        z += np.float32(s2 - s) * v
    return z


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def cosine(a, b) -> float:
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-30))
