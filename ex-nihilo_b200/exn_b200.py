"""Host-side mirror of ex-nihilo's DiT driver over libexn_b200.so.

The reference drives its DiT from Common Lisp (SBCL, not available here)
through three functions of src/cuda-dit.lisp and one loop of
src/generate.lisp; this module keeps their names, arguments and error
behaviour on top of the C ABI in include/exn_b200.h:

    upload_dit(path, device=0)                       (upload-dit path :device)  cuda-dit.lisp:52
    dit_velocity(d, context, p, latent, h, w, sigma,
                 prefix_key=None, ref=None)           (dit-velocity ...)         cuda-dit.lisp:137
    dit_release(d)                                    (dit-release d)            cuda-dit.lisp:99
    euler_steps(d, context, p, z, h, w, sigmas, ...)  generate's loop            generate.lisp:133-135

Errors are raised as ``ExnError`` carrying the library's message (the
reference signals Lisp errors, e.g. open-dit's list of bad tensors).
Arrays are numpy float32; latents channel-major (64, H, W).  Nothing here
computes: a missing library or device raises, there is no fallback.
"""
from __future__ import annotations

import ctypes
import hashlib
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("EXN_B200_LIB", os.path.join(HERE, "libexn_b200.so"))

# src/generate.lisp:7-9
TURBO_SIGMAS = (1.0, 0.978453, 0.95418, 0.926626, 0.89508, 0.845148, 0.704534, 0.414568, 0.0)

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
EXN_OK = 0
CODES = {1: "EINVAL", 2: "ECUDA", 3: "ESHAPE", 4: "ENOWEIGHTS", 5: "EIO", 6: "ETIMEOUT", 7: "ENOMEM",
         8: "EUNSUPPORTED"}


class ExnError(RuntimeError):
    def __init__(self, code, message):
        super().__init__("%s: %s" % (CODES.get(code, code), message))
        self.code = code


class Config(ctypes.Structure):
    _fields_ = [("width", ctypes.c_int), ("layers", ctypes.c_int), ("ffn", ctypes.c_int), ("latent", ctypes.c_int),
                ("context", ctypes.c_int), ("freq", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("device", ctypes.c_int)]


class EncConfig(ctypes.Structure):
    _fields_ = [("width", ctypes.c_int), ("layers", ctypes.c_int), ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int),
                ("ffn", ctypes.c_int), ("vocab", ctypes.c_int), ("theta", ctypes.c_double), ("device", ctypes.c_int)]


class Ref(ctypes.Structure):
    _fields_ = [("a", ctypes.c_int), ("latent", ctypes.POINTER(ctypes.c_float)), ("rh", ctypes.c_int),
                ("rw", ctypes.c_int)]


_lib = None


def lib():
    """The loaded libexn_b200.so (raises if it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ExnError(8, "%s is not built (python ex-nihilo_b200/build.py)" % LIB_PATH)
    L = ctypes.CDLL(LIB_PATH)
    H = ctypes.c_void_p
    fp = ctypes.POINTER(ctypes.c_float)
    vp = ctypes.c_void_p
    sigs = {
        "exn_abi_version": (ctypes.c_int, []),
        "exn_default_config": (None, [ctypes.POINTER(Config)]),
        "exn_open": (ctypes.c_int, [ctypes.POINTER(Config), ctypes.POINTER(H)]),
        "exn_close": (None, [H]),
        "exn_last_error": (ctypes.c_char_p, [H]),
        "exn_load_gguf": (ctypes.c_int, [H, ctypes.c_char_p]),
        "exn_check_gguf": (ctypes.c_int, [ctypes.POINTER(Config), ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]),
        "exn_load_tensor": (ctypes.c_int, [H, ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
                                           ctypes.POINTER(ctypes.c_int64), vp, ctypes.c_size_t]),
        "exn_load_synthetic": (ctypes.c_int, [H, ctypes.c_uint64]),
        "exn_weights_ready": (ctypes.c_int, [H]),
        "exn_velocity": (ctypes.c_int, [H, fp, ctypes.c_int, fp, ctypes.c_int, ctypes.c_int, ctypes.c_double,
                                        ctypes.c_uint64, ctypes.POINTER(Ref), fp]),
        "exn_generate": (ctypes.c_int, [H, fp, ctypes.c_int, fp, ctypes.c_int, ctypes.c_int,
                                        ctypes.POINTER(ctypes.c_double), ctypes.c_int, ctypes.c_uint64,
                                        ctypes.POINTER(Ref)]),
        "exn_generate_batch": (ctypes.c_int, [H, ctypes.c_int, fp, ctypes.c_int, fp, ctypes.c_int, ctypes.c_int,
                                              ctypes.POINTER(ctypes.c_double), ctypes.c_int]),
        "exn_generate_device": (ctypes.c_int, [H, ctypes.c_int, vp, ctypes.c_int, vp, ctypes.c_int, ctypes.c_int,
                                               ctypes.POINTER(ctypes.c_double), ctypes.c_int, vp]),
        "exn_sync": (ctypes.c_int, [H]),
        "exn_vae_open": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(H)]),
        "exn_vae_close": (None, [H]),
        "exn_vae_last_error": (ctypes.c_char_p, [H]),
        "exn_vae_load_safetensors": (ctypes.c_int, [H, ctypes.c_char_p]),
        "exn_vae_load_synthetic": (ctypes.c_int, [H, ctypes.c_uint64]),
        "exn_vae_weights_ready": (ctypes.c_int, [H]),
        "exn_vae_decode": (ctypes.c_int, [H, fp, ctypes.c_int, ctypes.c_int, fp]),
        "exn_vae_release": (ctypes.c_int, [H]),
        "exn_test_vae_last_ms": (ctypes.c_int, [H, ctypes.POINTER(ctypes.c_double)]),
        "exn_enc_default_config": (None, [ctypes.POINTER(EncConfig)]),
        "exn_enc_open": (ctypes.c_int, [ctypes.POINTER(EncConfig), ctypes.POINTER(H)]),
        "exn_enc_close": (None, [H]),
        "exn_enc_last_error": (ctypes.c_char_p, [H]),
        "exn_enc_load_gguf": (ctypes.c_int, [H, ctypes.c_char_p]),
        "exn_enc_load_synthetic": (ctypes.c_int, [H, ctypes.c_uint64]),
        "exn_enc_weights_ready": (ctypes.c_int, [H]),
        "exn_enc_states": (ctypes.c_int, [H, ctypes.POINTER(ctypes.c_int32), ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_int32), fp]),
        "exn_enc_states_device": (ctypes.c_int, [H, ctypes.POINTER(ctypes.c_int32), ctypes.c_int,
                                                 ctypes.POINTER(ctypes.c_int32), ctypes.c_int, vp, vp]),
        "exn_enc_release": (ctypes.c_int, [H]),
        "exn_test_enc_last_ms": (ctypes.c_int, [H, ctypes.POINTER(ctypes.c_double)]),
        "exn_test_enc_weights_digest": (ctypes.c_int, [H, ctypes.POINTER(ctypes.c_uint64)]),
        "exn_release": (ctypes.c_int, [H]),
        "exn_comm_unique_id": (ctypes.c_int, [vp]),
        "exn_comm_init": (ctypes.c_int, [H, vp, ctypes.c_int, ctypes.c_int]),
        "exn_comm_destroy": (ctypes.c_int, [H]),
        # testing entry points (include/exn_b200_testing.h)
        "exn_test_gemm": (ctypes.c_int, [H, vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
        "exn_test_gemm_q8": (ctypes.c_int, [H, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.POINTER(ctypes.c_double)]),
        "exn_test_gemm_i8": (ctypes.c_int, [H, vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.POINTER(ctypes.c_double)]),
        "exn_test_gemm_timed": (ctypes.c_int, [H, vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                               ctypes.POINTER(ctypes.c_double)]),
        "exn_test_attention": (ctypes.c_int, [H, vp, vp, vp, vp] + [ctypes.c_int] * 9),
        "exn_test_gemv": (ctypes.c_int, [H, ctypes.c_int, vp, vp, vp, vp] + [ctypes.c_int] * 6 +
                          [ctypes.POINTER(ctypes.c_double)]),
        "exn_test_attention_timed": (ctypes.c_int, [H, vp, vp, vp, vp] + [ctypes.c_int] * 10 +
                                     [ctypes.POINTER(ctypes.c_double)]),
        "exn_test_gemm_pairs": (ctypes.c_int, [H, ctypes.c_int]),
        "exn_test_comm_stats": (ctypes.c_int, [H, ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
                                               ctypes.POINTER(ctypes.c_double)]),
        "exn_test_attention_split": (ctypes.c_int, [H, ctypes.c_int, ctypes.c_int]),
        "exn_test_ln_mod": (ctypes.c_int, [H, vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
        "exn_test_qkv": (ctypes.c_int, [H, ctypes.c_int, vp, vp, vp, vp] + [ctypes.c_int] * 6),
        "exn_qkv_noalloc": (ctypes.c_int, [H, ctypes.c_int, vp, vp, vp, vp] + [ctypes.c_int] * 6),
        "exn_test_trace": (ctypes.c_int, [H, vp, ctypes.c_size_t]),
        "exn_test_weight_bf16": (ctypes.c_int, [H, ctypes.c_char_p, vp, ctypes.c_size_t]),
        "exn_test_synth_normal": (ctypes.c_int, [H, vp, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint32,
                                                 ctypes.c_double]),
        "exn_test_synth_q8": (ctypes.c_int, [H, vp, vp, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint32,
                                             ctypes.c_double]),
        "exn_test_weights_digest": (ctypes.c_int, [H, ctypes.POINTER(ctypes.c_uint64)]),
        "exn_test_last_profile": (ctypes.c_int, [H] + [ctypes.POINTER(ctypes.c_double)] * 4),
        "exn_test_last_barrier_ms": (ctypes.c_int, [H, ctypes.POINTER(ctypes.c_double)]),
        "exn_test_profile": (ctypes.c_int, [H, ctypes.c_int]),
        "exn_test_launch_count": (ctypes.c_longlong, [H]),
        "exn_test_last_call_ms": (ctypes.c_int, [H, ctypes.POINTER(ctypes.c_double)]),
        "exn_test_wait_probe": (ctypes.c_int, [H, ctypes.c_double]),
    }
    for name, (res, args) in sigs.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _f32(a, shape=None):
    a = np.ascontiguousarray(a, dtype=np.float32)
    if shape is not None and a.size != int(np.prod(shape)):
        raise ExnError(1, "array of %d floats, expected %s" % (a.size, shape))
    return a


def prefix_key_of(key) -> int:
    """A Lisp prefix key (any value compared with EQUAL: a prompt string, a
    list) as the ABI's nonzero 64-bit key; None is NIL (0)."""
    if key is None:
        return 0
    if isinstance(key, int) and 0 < key < 1 << 64:
        return key
    h = int.from_bytes(hashlib.blake2b(repr(key).encode(), digest_size=8).digest(), "little")
    return h or 1


def comm_unique_id() -> bytes:
    """An NCCL unique id (128 bytes) for exn_comm_init: made once, passed to every rank."""
    buf = ctypes.create_string_buffer(128)
    rc = lib().exn_comm_unique_id(buf)
    if rc != EXN_OK:
        raise ExnError(rc, lib().exn_last_error(None).decode(errors="replace"))
    return buf.raw


def default_config(**kw) -> Config:
    c = Config()
    lib().exn_default_config(ctypes.byref(c))
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def check_gguf(path, **shape) -> None:
    """open-dit (src/weights.lisp:47-61) without a device: raises ExnError
    listing every problem."""
    c = default_config(**shape)
    buf = ctypes.create_string_buffer(8192)
    rc = lib().exn_check_gguf(ctypes.byref(c), str(path).encode(), buf, len(buf))
    if rc != EXN_OK:
        raise ExnError(rc, buf.value.decode(errors="replace"))


class Dit:
    """A DiT on one CUDA device: the reference's GDIT structure."""

    def __init__(self, device=0, **shape):
        self.cfg = default_config(device=device, **shape)
        h = ctypes.c_void_p()
        rc = lib().exn_open(ctypes.byref(self.cfg), ctypes.byref(h))
        if rc != EXN_OK:
            raise ExnError(rc, lib().exn_last_error(None).decode(errors="replace"))
        self.h = h

    # -- plumbing
    def _ck(self, rc):
        if rc != EXN_OK:
            raise ExnError(rc, lib().exn_last_error(self.h).decode(errors="replace"))

    def close(self):
        if getattr(self, "h", None):
            lib().exn_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # -- weights
    def load_gguf(self, path):
        self._ck(lib().exn_load_gguf(self.h, str(path).encode()))

    def load_tensor(self, name, ggml_type, dims, data: np.ndarray):
        d = (ctypes.c_int64 * len(dims))(*dims)
        data = np.ascontiguousarray(data)
        self._ck(lib().exn_load_tensor(self.h, name.encode(), ggml_type, len(dims), d,
                                       data.ctypes.data_as(ctypes.c_void_p), data.nbytes))

    def load_synthetic(self, seed=1):
        self._ck(lib().exn_load_synthetic(self.h, seed))

    def ready(self) -> bool:
        return lib().exn_weights_ready(self.h) == EXN_OK

    # -- steps
    def _ref(self, ref):
        if ref is None:
            return None, None
        a, rlat, rh, rw = ref
        rlat = _f32(rlat, (self.cfg.latent, rh, rw))
        return Ref(a, _fp(rlat), rh, rw), rlat

    def velocity(self, context, p, latent, h, w, sigma, prefix_key=None, ref=None):
        ctx = _f32(context, (p, self.cfg.context))
        lat = _f32(latent, (self.cfg.latent, h, w))
        v = np.empty((self.cfg.latent, h, w), dtype=np.float32)
        r, keep = self._ref(ref)
        self._ck(lib().exn_velocity(self.h, _fp(ctx), p, _fp(lat), h, w, float(sigma), prefix_key_of(prefix_key),
                                    ctypes.byref(r) if r is not None else None, _fp(v)))
        del keep
        return v

    def generate(self, context, p, z, h, w, sigmas=TURBO_SIGMAS, prefix_key=None, ref=None):
        ctx = _f32(context, (p, self.cfg.context))
        zz = np.array(_f32(z, (self.cfg.latent, h, w)), copy=True).reshape(self.cfg.latent, h, w)
        s = (ctypes.c_double * len(sigmas))(*sigmas)
        r, keep = self._ref(ref)
        self._ck(lib().exn_generate(self.h, _fp(ctx), p, _fp(zz), h, w, s, len(sigmas), prefix_key_of(prefix_key),
                                    ctypes.byref(r) if r is not None else None))
        del keep
        return zz

    def generate_batch(self, contexts, p, z, h, w, sigmas=TURBO_SIGMAS):
        b = int(np.asarray(z).shape[0])
        ctx = _f32(contexts, (b, p, self.cfg.context))
        zz = np.array(_f32(z, (b, self.cfg.latent, h, w)), copy=True).reshape(b, self.cfg.latent, h, w)
        s = (ctypes.c_double * len(sigmas))(*sigmas)
        self._ck(lib().exn_generate_batch(self.h, b, _fp(ctx), p, _fp(zz), h, w, s, len(sigmas)))
        return zz

    def generate_device(self, batch, d_contexts, p, d_z, h, w, sigmas=TURBO_SIGMAS, stream=0):
        """Device pointers (ints) in, ordered on STREAM (an int cudaStream_t; 0 is CUDA's default stream)."""
        s = (ctypes.c_double * len(sigmas))(*sigmas)
        self._ck(lib().exn_generate_device(self.h, batch, ctypes.c_void_p(d_contexts), p, ctypes.c_void_p(d_z), h, w,
                                           s, len(sigmas), ctypes.c_void_p(stream or 0)))

    def sync(self):
        self._ck(lib().exn_sync(self.h))

    def release(self):
        self._ck(lib().exn_release(self.h))

    def comm_init(self, uid: bytes, rank: int, world: int):
        """Share this picture's rows with WORLD ranks (sequence parallelism, NCCL all-to-all)."""
        buf = ctypes.create_string_buffer(bytes(uid), 128)
        self._ck(lib().exn_comm_init(self.h, buf, rank, world))

    def comm_destroy(self):
        self._ck(lib().exn_comm_destroy(self.h))

    def profile(self, on=True):
        self._ck(lib().exn_test_profile(self.h, 1 if on else 0))

    def last_profile(self):
        g, a, o, u = ctypes.c_double(), ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
        self._ck(lib().exn_test_last_profile(self.h, ctypes.byref(g), ctypes.byref(a), ctypes.byref(o), ctypes.byref(u)))
        b = ctypes.c_double()
        self._ck(lib().exn_test_last_barrier_ms(self.h, ctypes.byref(b)))
        return dict(gemm_ms=g.value, attn_ms=a.value, other_ms=o.value, gateup_ms=u.value, barrier_ms=b.value)

    def launch_count(self):
        return int(lib().exn_test_launch_count(self.h))

    def comm_stats(self):
        """(waits for a queued NCCL call, 50 us sleeps in them, seconds) since open."""
        n, z, t = ctypes.c_longlong(), ctypes.c_longlong(), ctypes.c_double()
        self._ck(lib().exn_test_comm_stats(self.h, ctypes.byref(n), ctypes.byref(z), ctypes.byref(t)))
        return n.value, z.value, t.value

    def last_call_ms(self):
        """Device time of the last velocity / generate call, inputs in HBM (ms)."""
        ms = ctypes.c_double()
        self._ck(lib().exn_test_last_call_ms(self.h, ctypes.byref(ms)))
        return ms.value


class Vae:
    """The VAE decoder on one CUDA device: the reference's GVAE structure (src/cuda-vae.lisp:10-13)."""

    def __init__(self, device=0):
        h = ctypes.c_void_p()
        rc = lib().exn_vae_open(device, ctypes.byref(h))
        if rc != EXN_OK:
            raise ExnError(rc, lib().exn_vae_last_error(None).decode(errors="replace"))
        self.h = h

    def _ck(self, rc):
        if rc != EXN_OK:
            raise ExnError(rc, lib().exn_vae_last_error(self.h).decode(errors="replace"))

    def close(self):
        if getattr(self, "h", None):
            lib().exn_vae_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def load_safetensors(self, path):
        self._ck(lib().exn_vae_load_safetensors(self.h, str(path).encode()))

    def load_synthetic(self, seed=1):
        self._ck(lib().exn_vae_load_synthetic(self.h, seed))

    def decode(self, latent, h, w):
        """LATENT (64 x h x w, denormalised) -> RGBA (16h, 16w, 4) in -1 .. 1."""
        z = _f32(latent, (64, h, w))
        out = np.empty((16 * h, 16 * w, 4), dtype=np.float32)
        self._ck(lib().exn_vae_decode(self.h, _fp(z), h, w, _fp(out)))
        return out

    def release(self):
        self._ck(lib().exn_vae_release(self.h))

    def last_ms(self):
        ms = ctypes.c_double()
        self._ck(lib().exn_test_vae_last_ms(self.h, ctypes.byref(ms)))
        return ms.value


class Encoder:
    """The prompt encoder (Qwen3-VL-8B's text model) on one CUDA device: what load-encoder returns
    (src/encoder.lisp:41-48).  SHAPE overrides fields of exn_enc_default_config (width, layers,
    heads, kv_heads, ffn, vocab, theta)."""

    def __init__(self, device=0, **shape):
        cfg = EncConfig()
        lib().exn_enc_default_config(ctypes.byref(cfg))
        for k, v in shape.items():
            setattr(cfg, k, v)
        cfg.device = device
        h = ctypes.c_void_p()
        rc = lib().exn_enc_open(ctypes.byref(cfg), ctypes.byref(h))
        if rc != EXN_OK:
            raise ExnError(rc, lib().exn_enc_last_error(None).decode(errors="replace"))
        self.h = h
        self.cfg = cfg

    def _ck(self, rc):
        if rc != EXN_OK:
            raise ExnError(rc, lib().exn_enc_last_error(self.h).decode(errors="replace"))

    def close(self):
        if getattr(self, "h", None):
            lib().exn_enc_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def load_gguf(self, path):
        self._ck(lib().exn_enc_load_gguf(self.h, str(path).encode()))

    def load_synthetic(self, seed=1):
        self._ck(lib().exn_enc_load_synthetic(self.h, seed))

    def states(self, ids, positions=None):
        """encoder-states: (n, width) float32, the last block's output before the final norm.
        POSITIONS: (n, 3) ints (t, h, w) or None for a text prompt's (i, i, i)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32).ravel()
        n = len(ids)
        pos = None
        if positions is not None:
            pos = np.ascontiguousarray(positions, dtype=np.int32)
            if pos.shape != (n, 3):
                raise ExnError(1, "positions must be (n, 3), got %s" % (pos.shape,))
        out = np.empty((n, self.cfg.width), dtype=np.float32)
        ip = ctypes.POINTER(ctypes.c_int32)
        self._ck(lib().exn_enc_states(self.h, ids.ctypes.data_as(ip), n,
                                      pos.ctypes.data_as(ip) if pos is not None else None, _fp(out)))
        return out

    def states_device(self, ids, d_states, positions=None, skip=0, stream=None):
        """encode-prompt's states into device memory (a pointer, e.g. a torch tensor's data_ptr()):
        rows SKIP.. of the states, ready for Dit.generate_device as its context."""
        ids = np.ascontiguousarray(ids, dtype=np.int32).ravel()
        n = len(ids)
        pos = None
        if positions is not None:
            pos = np.ascontiguousarray(positions, dtype=np.int32)
            if pos.shape != (n, 3):
                raise ExnError(1, "positions must be (n, 3), got %s" % (pos.shape,))
        ip = ctypes.POINTER(ctypes.c_int32)
        self._ck(lib().exn_enc_states_device(self.h, ids.ctypes.data_as(ip), n,
                                             pos.ctypes.data_as(ip) if pos is not None else None, skip,
                                             ctypes.c_void_p(d_states), ctypes.c_void_p(stream)))

    def release(self):
        self._ck(lib().exn_enc_release(self.h))

    def last_ms(self):
        ms = ctypes.c_double()
        self._ck(lib().exn_test_enc_last_ms(self.h, ctypes.byref(ms)))
        return ms.value

    def weights_digest(self):
        d = ctypes.c_uint64()
        self._ck(lib().exn_test_enc_weights_digest(self.h, ctypes.byref(d)))
        return d.value


# ---- the reference's names

def upload_dit(path, device=0, **shape) -> Dit:
    """(upload-dit path :device device), src/cuda-dit.lisp:52-86."""
    d = Dit(device=device, **shape)
    try:
        d.load_gguf(path)
    except Exception:
        d.close()
        raise
    return d


def dit_velocity(d: Dit, context, p, latent, h, w, sigma, prefix_key=None, ref=None):
    """(dit-velocity d context p latent h w sigma :prefix-key :ref), src/cuda-dit.lisp:137-243."""
    return d.velocity(context, p, latent, h, w, sigma, prefix_key=prefix_key, ref=ref)


def dit_release(d: Dit):
    """(dit-release d), src/cuda-dit.lisp:99-108."""
    d.release()


def euler_steps(d: Dit, context, p, z, h, w, sigmas=TURBO_SIGMAS, prefix_key=None, ref=None):
    """generate's loop (src/generate.lisp:133-135) with the update fused on the device."""
    return d.generate(context, p, z, h, w, sigmas, prefix_key=prefix_key, ref=ref)


def upload_vae(path, device=0) -> Vae:
    """(upload-vae path :device device), src/cuda-vae.lisp:15-27 (the decoder's tensors)."""
    v = Vae(device)
    try:
        v.load_safetensors(path)
    except Exception:
        v.close()
        raise
    return v


def vae_decode(v: Vae, latent, h, w):
    """(vae-decode v latent h w), src/cuda-vae.lisp:94-136: RGBA rows, channels last."""
    return v.decode(latent, h, w)


def vae_release(v: Vae):
    """(vae-release v), src/cuda-vae.lisp:29-33."""
    v.release()


def load_encoder(path, device=0, **shape) -> Encoder:
    """(load-encoder path :device device), src/encoder.lisp:41-48, on the B200."""
    e = Encoder(device=device, **shape)
    try:
        e.load_gguf(path)
    except Exception:
        e.close()
        raise
    return e


def encoder_states(e: Encoder, ids, positions=None):
    """(encoder-states model ids :rope (mrope-table positions ...)), src/encoder.lisp:143-183."""
    return e.states(ids, positions)
