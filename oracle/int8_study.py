"""Numerics study, not product code: how far int8 activation schemes put the
DiT from the fp32 oracle, next to bf16 operands.

Test infrastructure only (it patches the oracle's `linear`).  Three ways to
feed a GEMM of n >= 16 rows (src/cuda-dit.lisp:115-130 sends those through
int8 when `*int8*` is on, src/cuda-dit.lisp:110-113):

  bf16   both operands rounded to bf16, products summed exactly (the shipped
         tcgen05 kind::f16 GEMMs)
  ref8   the reference's default: activations quantised to Q8_0 by blocks of
         32 along K (fp16 scale = amax / 127, round to nearest), weights as
         loaded (exact Q8_0), per-block integer dots scaled and summed
  tok8   the only int8 form one tcgen05 kind::i8 accumulation per tile can
         take: one scale per activation row and one per weight row

Usage: python oracle/int8_study.py [layers]   (width 512, FFN 1536, 32 text
rows, 16 x 16 latent, sigma 1; prints velocity and 8-step latent errors)
"""
import sys

import numpy as np

sys.path.insert(0, __import__("os").path.dirname(__import__("os").path.dirname(__file__)))
import oracle.dit_oracle as O  # noqa: E402


def to_bf16(a):
    """Round-to-nearest-even to bf16, returned as float32."""
    u = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def quant_rows(x, blk, fp16_scale):
    """x quantised to int8 by blocks of BLK along the row, dequantised back."""
    n, k = x.shape
    xb = x.reshape(n, k // blk, blk).astype(np.float32)
    d = np.abs(xb).max(-1, keepdims=True) / np.float32(127.0)
    if fp16_scale:
        d = d.astype(np.float16).astype(np.float32)
    safe = np.where(d > 0, d, 1)
    q = np.clip(np.rint(xb / safe), -127, 127) * (d > 0)
    return (q * d).reshape(n, k)


def make_linear(mode, base):
    def lin(x, w):
        if x.shape[0] < 16:
            return base(x, w)
        if mode == "bf16":
            a, b = to_bf16(x), to_bf16(w)
        elif mode == "ref8":
            a, b = quant_rows(x, 32, True), w
        elif mode == "tok8":
            a, b = quant_rows(x, x.shape[1], False), quant_rows(w, w.shape[1], False)
        else:
            raise ValueError(mode)
        return a.astype(np.float64) @ b.astype(np.float64).T
    return lin


def main(layers=6):
    sh = O.Shape(width=512, layers=layers, ffn=1536, context=512)
    wt = O.SynthWeights.make(sh, 1)
    ctx, z = O.synth_inputs(sh, 32, 16, 16)
    ctx, z = ctx[0], z[0]
    base = O.linear
    try:
        v0 = O.forward(wt, sh, ctx, z, 1.0)
        z0 = O.euler(wt, sh, ctx, z)
        for mode in ("bf16", "ref8", "tok8"):
            O.linear = make_linear(mode, base)
            v = O.forward(wt, sh, ctx, z, 1.0)
            zz = O.euler(wt, sh, ctx, z)
            O.linear = base
            print("%-5s velocity rel-L2 %.4f cosine %.6f | 8-step latent rel-L2 %.4f cosine %.6f" % (
                mode, O.rel_l2(v, v0), O.cosine(v.ravel(), v0.ravel()),
                O.rel_l2(zz, z0), O.cosine(zz.ravel(), z0.ravel())))
    finally:
        O.linear = base


if __name__ == "__main__":
    main(int(sys.argv[1]) if len(sys.argv) > 1 else 6)
