"""Build libexn_b200.so in place (next to this file) for sm_100a.

    python ex-nihilo_b200/build.py [--force]

Each source is compiled by nvcc with ``-gencode arch=compute_100a,code=sm_100a``
into ``_build/`` (objects rebuilt when the source or any header is newer) and
linked into a shared library with the CUDA runtime linked statically, so the
library needs only the driver at run time.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libexn_b200.so")
SOURCES = ["gemm.cu", "gemm_q8.cu", "gemm_thin.cu", "conv.cu", "attention.cu", "elementwise.cu", "vae.cu", "encoder.cu", "noalloc.cu",
           "dit.cpp", "vae.cpp", "encoder.cpp", "gguf.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def flags():
    return ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3,-Wall", "-I", os.path.join(ROOT, "include"),
                   "-I", CSRC, "--expt-relaxed-constexpr"]


def _newest_header():
    hs = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0)


def _compile(src, force):
    s = os.path.join(CSRC, src)
    o = os.path.join(BUILD, src + ".o")
    if not force and os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), _newest_header()):
        return o, None
    cmd = [nvcc()] + flags() + ["-x", "cu" if src.endswith(".cu") else "c++", "-c", s, "-o", o]
    if not src.endswith(".cu"):
        cmd = [nvcc()] + flags() + ["-c", s, "-o", o]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return o, "%s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr)
    return o, None


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, force), SOURCES))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("build failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    try:
        build(force=a.force, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
