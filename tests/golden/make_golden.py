"""Generate the golden vectors in this directory by running the reference's own
numpy DiT, ``inspect/ref_dit.py`` of ex-nihilo, on synthetic inputs.

    python tests/golden/make_golden.py --ref-dir <ex-nihilo>/inspect [--full]

The DiT cases run ``inspect/ref_dit.py``; the VAE case (``vae_small``) runs ``inspect/ref_vae.py``.

For each case it

1. makes the synthetic DiT with ``oracle.dit_oracle.SynthWeights`` (Q8_0),
2. writes it as a real ``qwen_image`` GGUF with gguf-py and reads it back
   through ref_dit.py's own ``Weights`` (GGUFReader + gguf dequantize),
3. patches ref_dit's module constants W/HEADS/FFN/LAYERS to the case's shape
   and runs its ``forward`` (the velocity, ``txt.f32`` and ``blk0.f32`` dumps
   and the per-block ``|x|`` lines it prints),
4. for the Euler cases, steps ``z += (s' - s) v`` over the Turbo sigmas as
   src/generate.lisp:133-135 does, each v from ref_dit.forward,

and stores the outputs with checksums of the weights and inputs in
``<case>.npz``.  The reference tree is read only here, never by the tests or
the GPU runs; they use the stored vectors.
"""
from __future__ import annotations

import argparse
import contextlib
import hashlib
import importlib.util
import io
import json
import os
import re
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle import dit_oracle as O  # noqa: E402
from oracle.synth_gguf import write_gguf  # noqa: E402

CASES = {
    # small: 2 heads, 2 blocks, non-square 4 x 6 latent, 8 text rows of width 256
    "tiny": dict(shape=dict(width=256, layers=2, ffn=768, context=256), p=8, h=4, w=6, sigma=0.7),
    # BASELINE config 1 with the reference's block math: D=2560 (20 heads), FFN 7680, one block,
    # 32 text rows of 4096, a 16 x 16 latent, t = 500
    "cfg1": dict(shape=dict(width=2560, layers=1, ffn=7680, context=4096), p=32, h=16, w=16, sigma=0.5),
    # the tiny DiT through the eight Turbo steps
    "tiny_euler": dict(shape=dict(width=256, layers=2, ffn=768, context=256), p=8, h=4, w=6, euler=True),
    # a 3-block D=512 DiT, 12 text rows, 8 x 8 latent, eight steps
    "small_euler": dict(shape=dict(width=512, layers=3, ffn=1536, context=512), p=12, h=8, w=8, euler=True),
}
FULL = {
    # the full 32-block D=4096 DiT at 1024^2 (64 x 64 latent), 128 text rows, 8 steps
    "cfg2_euler": dict(shape=dict(), p=128, h=64, w=64, euler=True),
    # 1536 x 1024 (a 64 x 96 latent, a non-square RoPE grid), 256 text rows, 8 steps
    "cfg3_euler": dict(shape=dict(), p=256, h=64, w=96, euler=True),
}


VAE_CASES = {
    # the decoder on an 8 x 8 latent (a 128 x 128 picture): every stage, the middle attention over 64 pixels
    "vae_small": dict(h=8, w=8),
}


def run_vae_case(ref_dir, name, case, outdir):
    """The reference's own inspect/ref_vae.py decoding a synthetic latent with the oracle's synthetic
    decoder weights, written as a real BF16 safetensors file and read back through ref_vae's ST."""
    from oracle import vae_oracle as V
    spec = importlib.util.spec_from_file_location("ref_vae", os.path.join(ref_dir, "ref_vae.py"))
    RV = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(RV)
    t0 = time.time()
    sw = V.SynthVae(1)
    z = O.synth_normal(0, 3000, (64, case["h"], case["w"]))
    h = hashlib.sha256()
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "vae.safetensors")
        V.write_safetensors(path, [(n, sw(n)) for n, _ in sw.spec])
        for n, _ in sw.spec:
            h.update(sw(n).tobytes())
        with contextlib.redirect_stdout(io.StringIO()):
            rgba = RV.decode(RV.ST(path), z)
    np.savez(os.path.join(outdir, name + ".npz"), rgba=rgba,
             meta=json.dumps(dict(case=name, h=case["h"], w=case["w"], weight_seed=1, latent="synth_normal(0, 3000)",
                                  reference="inspect/ref_vae.py decode, BF16 safetensors")),
             weights_sha256=np.array(h.hexdigest()), latent_sha256=np.array(hashlib.sha256(z.tobytes()).hexdigest()))
    print("%s: %.1fs" % (name, time.time() - t0), flush=True)


def load_ref(ref_dir):
    spec = importlib.util.spec_from_file_location("ref_dit", os.path.join(ref_dir, "ref_dit.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def weights_digest(sw: O.SynthWeights) -> str:
    h = hashlib.sha256()
    for name, _ in O.expected_tensors(sw.shape):
        if name in sw.vec:
            h.update(sw.vec[name].tobytes())
        else:
            qs, d = sw.q8[name]
            h.update(qs.tobytes())
            h.update(d.tobytes())
    return h.hexdigest()


def run_case(R, name, case, outdir):
    sh = O.Shape(**case["shape"])
    t0 = time.time()
    sw = O.SynthWeights.make(sh, seed=1)
    ctx, lat = O.synth_inputs(sh, case["p"], case["h"], case["w"], seed=0)
    ctx, lat = ctx[0], lat[0]
    R.W, R.HEADS, R.FFN, R.LAYERS = sh.width, sh.heads, sh.ffn, sh.layers
    out = dict(meta=json.dumps(dict(case=name, shape=case["shape"], p=case["p"], h=case["h"], w=case["w"],
                                    sigma=case.get("sigma"), weight_seed=1, input_seed=0,
                                    sigmas=list(O.TURBO_SIGMAS) if case.get("euler") else None,
                                    generator="oracle.dit_oracle synth_* (splitmix64, Irwin-Hall 4)",
                                    reference="inspect/ref_dit.py forward, gguf-py 0.19.0")),
               weights_sha256=np.array(weights_digest(sw)),
               ctx_sha256=np.array(hashlib.sha256(ctx.tobytes()).hexdigest()),
               lat_sha256=np.array(hashlib.sha256(lat.tobytes()).hexdigest()))
    with tempfile.TemporaryDirectory() as td:
        path = os.path.join(td, "dit.gguf")
        write_gguf(path, sw)
        wt = R.Weights(path)
        if not case.get("euler"):
            buf = io.StringIO()
            with contextlib.redirect_stdout(buf):
                v = R.forward(wt, ctx, lat, case["sigma"], dump=td)
            rms = [float(m) for m in re.findall(r"block \d+: \|x\| (\S+)", buf.getvalue())]
            txt = np.fromfile(os.path.join(td, "txt.f32"), dtype=np.float32).reshape(case["p"], sh.width)
            blk0 = np.fromfile(os.path.join(td, "blk0.f32"), dtype=np.float32).reshape(-1, sh.width)
            n = blk0.shape[0]
            if n * sh.width > 200_000:   # keep the fixture small: every text row, every 8th image row
                rows = np.concatenate([np.arange(case["p"]), np.arange(case["p"], n, 8)])
            else:
                rows = np.arange(n)
            out.update(v=v, txt=txt, blk0_rows=rows, blk0=blk0[rows], block_rms=np.array(rms))
        else:
            z = lat.copy()
            vs = []
            for s, s2 in zip(O.TURBO_SIGMAS[:-1], O.TURBO_SIGMAS[1:]):
                with contextlib.redirect_stdout(io.StringIO()):
                    v = R.forward(wt, ctx, z, s)
                vs.append(v)
                z = z + np.float32(s2 - s) * v
                z = z.astype(np.float32)
                print("  %s: sigma %.6f done, %.0fs" % (name, s, time.time() - t0), flush=True)
            out.update(z=z, v_first=vs[0], v_last=vs[-1])
    np.savez(os.path.join(outdir, name + ".npz"), **out)
    print("%s: %.1fs" % (name, time.time() - t0), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-dir", default=os.environ.get("EXN_REF_INSPECT"),
                    help="the reference tree's inspect/ directory (holds ref_dit.py); or set EXN_REF_INSPECT")
    ap.add_argument("--full", action="store_true", help="also the full D=4096 8-step cases (tens of minutes each)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    if not args.ref_dir:
        ap.error("--ref-dir (or EXN_REF_INSPECT) is required: the reference's inspect/ directory")
    R = load_ref(args.ref_dir)
    cases = dict(CASES)
    if args.full:
        cases.update(FULL)
    for name, case in cases.items():
        if args.only and name not in args.only.split(","):
            continue
        run_case(R, name, case, HERE)
    for name, case in VAE_CASES.items():
        if args.only and name not in args.only.split(","):
            continue
        run_vae_case(args.ref_dir, name, case, HERE)


if __name__ == "__main__":
    main()
