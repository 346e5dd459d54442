"""Single sm_100a kernels through the C ABI's testing entry points
(include/exn_b200_testing.h), on the cases of the reference's own kernel
tests (inspect/metal-kernels-test.lisp:91-146) and larger ones."""
import numpy as np
import pytest

import exn_b200 as E
from oracle import dit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TINY = dict(width=256, layers=2, ffn=768, context=256)


@pytest.fixture(scope="module")
def dit():
    d = E.Dit(**TINY)
    d.load_synthetic(1)
    yield d
    d.close()


def bf16(a):
    return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


@pytest.mark.parametrize("m,n,k", [(1, 64, 64), (100, 256, 256), (128, 256, 4096), (300, 512, 192),
                                   (1000, 768, 1024), (4224, 12288, 4096), (513, 64, 4096)])
def test_gemm_matches_fp64(dit, m, n, k):
    g = torch.Generator().manual_seed(m * 7 + n + k)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16)
    b = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
    ad, bd = a.cuda(), b.cuda()
    c = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    dit._ck(E.lib().exn_test_gemm(dit.h, ad.data_ptr(), bd.data_ptr(), c.data_ptr(), m, n, k))
    ref = (ad.double() @ bd.double().T)
    err = (c.double() - ref).abs().max().item() / ref.abs().max().item()
    assert torch.isfinite(c).all()
    assert err < 1e-5, err


@pytest.mark.parametrize("epi_shape", [(300, 512, 4096), (1088, 4096, 4096), (513, 12288, 4096),
                                       (576, 4096, 4096)])
def test_gemm_tile_shapes_are_bit_identical(dit, epi_shape):
    """256 x 256 tiles on CTA pairs (mode 2), 128-row tiles of one CTA (mode 0) and the default
    (mode 1: pairs, or 128 x 64 one-CTA tiles where pair tiles would not fill one round -- 300 and
    576 rows here) give every output element the same bits (the same k-order of the same MMAs), so
    a rank may pick any without changing a row."""
    m, n, k = epi_shape
    g = torch.Generator().manual_seed(m + n)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    b = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16).cuda()
    outs = []
    try:
        for pairs in (1, 2, 0):
            dit._ck(E.lib().exn_test_gemm_pairs(dit.h, pairs))
            c = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
            dit._ck(E.lib().exn_test_gemm(dit.h, a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k))
            outs.append(c)
    finally:
        dit._ck(E.lib().exn_test_gemm_pairs(dit.h, 1))
    assert torch.isfinite(outs[0]).all()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def q8_weights(n, k, seed):
    """Random Q8_0 weights: int8 q in [-127, 127] and fp16 block scales, with their bf16 slab."""
    g = torch.Generator().manual_seed(seed)
    qs = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int32).to(torch.int8)
    d = (torch.rand(n, k // 32, generator=g) * 0.002 + 1e-4).to(torch.float16)
    w = (qs.float() * d.float().repeat_interleave(32, dim=1)).to(torch.bfloat16)
    return qs, d, w


@pytest.mark.parametrize("m,n,k", [(100, 256, 256), (300, 512, 192), (1000, 768, 1024), (4224, 1024, 4096)])
def test_gemm_q8_equals_the_bf16_slab(dit, m, n, k):
    """The GEMM that converts Q8_0 weights in shared memory gives the same bits as the GEMM on the
    load-time bf16 slab of the same weights (each value round-to-nearest bf16 of q * d)."""
    qs, d, w = q8_weights(n, k, m + n)
    g = torch.Generator().manual_seed(k)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    c0 = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    c1 = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    dit._ck(E.lib().exn_test_gemm(dit.h, a.data_ptr(), w.cuda().data_ptr(), c0.data_ptr(), m, n, k))
    qd, dd = qs.cuda(), d.cuda()
    dit._ck(E.lib().exn_test_gemm_q8(dit.h, a.data_ptr(), qd.data_ptr(), dd.data_ptr(), c1.data_ptr(), m, n, k, 0,
                                     None))
    assert torch.isfinite(c1).all()
    assert torch.equal(c0, c1)


@pytest.mark.parametrize("m,n,k", [(100, 256, 128), (300, 512, 384), (1000, 768, 4096)])
def test_gemm_i8_matches_exact_integer_product(dit, m, n, k):
    """The int8 (kind::i8) GEMM: s32 accumulation is exact, so with unit scales it equals the integer
    product exactly, and with scales it is that product times sa[row] sb[col] (fp32 roundings only)."""
    g = torch.Generator().manual_seed(m + k)
    a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int32)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int32)
    exact = (a.double() @ b.double().T)
    sa = torch.rand(m, generator=g) + 0.5
    sb = torch.rand(n, generator=g) + 0.5
    ad, bd = a.to(torch.int8).cuda(), b.to(torch.int8).cuda()
    for scaled in (False, True):
        s_a = (sa if scaled else torch.ones(m)).float().cuda()
        s_b = (sb if scaled else torch.ones(n)).float().cuda()
        c = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
        dit._ck(E.lib().exn_test_gemm_i8(dit.h, ad.data_ptr(), bd.data_ptr(), s_a.data_ptr(), s_b.data_ptr(),
                                         c.data_ptr(), m, n, k, 0, None))
        want = exact * s_a.double().cpu()[:, None] * s_b.double().cpu()[None, :]
        got = c.double().cpu()
        if scaled:
            assert ((got - want).abs() / want.abs().clamp_min(1.0)).max().item() < 1e-6
        else:
            assert torch.equal(got, exact.float().double())   # the exact s32 sum, rounded once to fp32


def attention_ref(q, k, v, q0, p, l, b0, b1, heads):
    """fp64 masked softmax attention on the (already bf16-rounded) inputs."""
    qq = q.double().reshape(q.shape[0], heads, 128)
    kk = k[:l].double().reshape(l, heads, 128)
    vv = v[:l].double().reshape(l, heads, 128)
    lim = torch.as_tensor(O.xa_lim(np.arange(q0, q0 + q.shape[0]), p, l, b0, b1))
    mask = torch.arange(l)[None, :] > lim[:, None]
    s = torch.einsum("qhd,khd->hqk", qq, kk) / np.sqrt(128.0)
    s = s.masked_fill(mask[None], float("-inf"))
    return torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), vv).reshape(q.shape[0], heads * 128)


# (name, batch, nq, q0, p, l, b0, b1, heads): the first three are metal-kernels-test.lisp:144-146
CASES = [
    ("first pass: prompt causal, image all", 1, 77, 0, 20, 77, 20, 20, 32),
    ("image after a cached prompt", 1, 70, 33, 33, 103, 33, 33, 32),
    ("reference picture in the prompt", 1, 90, 0, 40, 90, 12, 30, 32),
    ("two samples, tile tails", 2, 300, 0, 40, 300, 0, 0, 4),
    ("cached, several key tiles", 2, 513, 128, 128, 641, 0, 0, 2),
    ("1024^2 first step, 2 heads", 1, 4224, 0, 128, 4224, 0, 0, 2),
    ("edit layout", 1, 700, 0, 300, 700, 8, 264, 2),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_attention_mask_cases(dit, case):
    _, batch, nq, q0, p, l, b0, b1, heads = case
    w = heads * 128
    kv_rows = l + 5
    g = torch.Generator().manual_seed(nq + l)
    q = ((torch.rand(batch, nq, w, generator=g) * 4 - 2)).to(torch.bfloat16)
    k = ((torch.rand(batch, kv_rows, w, generator=g) * 4 - 2)).to(torch.bfloat16)
    v = ((torch.rand(batch, kv_rows, w, generator=g) * 2 - 1)).to(torch.bfloat16)
    qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
    out = torch.full((batch, nq, w), float("nan"), dtype=torch.bfloat16, device="cuda")
    dit._ck(E.lib().exn_test_attention(dit.h, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), out.data_ptr(),
                                       batch, nq, q0, p, l, b0, b1, heads, kv_rows))
    got = out.float().cpu()
    for b in range(batch):
        want = attention_ref(q[b], k[b], v[b], q0, p, l, b0, b1, heads)
        err = (got[b].double() - want).abs().max().item()
        # the reference's bound for half P (metal-kernels-test.lisp:5-8); bf16 P rounds at 2^-9 and
        # the output itself is bf16 (|v| < 1)
        assert err < 3e-3 + 2 ** -8, (b, err)


@pytest.mark.parametrize("nq", [300, 700])
def test_attention_work_splits_are_bit_identical(dit, nq):
    """The attention kernel's work splits (two-tile CTAs only; one-tile CTAs only; two-tile CTAs with a
    short last round run as one-tile CTAs, forced here by planning for fewer SMs) give every query row the
    same bits, also for a row count that is not a multiple of 256."""
    batch, q0, p, heads = 1, 0, 40, 4
    l = nq
    w = heads * 128
    g = torch.Generator().manual_seed(nq)
    q = ((torch.rand(batch, nq, w, generator=g) * 4 - 2)).to(torch.bfloat16).cuda()
    k = ((torch.rand(batch, l, w, generator=g) * 4 - 2)).to(torch.bfloat16).cuda()
    v = ((torch.rand(batch, l, w, generator=g) * 2 - 1)).to(torch.bfloat16).cuda()
    items = -(-nq // 256) * heads * batch           # two-tile work items
    plan = items - 2                                # a last round of 2 items: split into 4 one-tile CTAs
    assert 0 < items % plan and 2 * (items % plan) <= plan
    outs = []
    try:
        for mode, sms in [(0, 0), (1, 0), (2, plan)]:
            dit._ck(E.lib().exn_test_attention_split(dit.h, mode, sms))
            o = torch.full((batch, nq, w), float("nan"), dtype=torch.bfloat16, device="cuda")
            dit._ck(E.lib().exn_test_attention(dit.h, q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                               batch, nq, q0, p, l, 0, 0, heads, l))
            outs.append(o.view(torch.int16).cpu())
    finally:
        dit._ck(E.lib().exn_test_attention_split(dit.h, 2, 0))
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(outs[0], outs[2])


def test_attention_timed_equals_single_launch(dit):
    """exn_test_attention_timed queues the same launch REPS times: the output is the single launch's,
    bit for bit, and the mean time is positive."""
    import ctypes
    batch, nq, q0, p, heads = 1, 700, 0, 300, 2
    w = heads * 128
    g = torch.Generator().manual_seed(5)
    q = ((torch.rand(batch, nq, w, generator=g) * 4 - 2)).to(torch.bfloat16).cuda()
    k = ((torch.rand(batch, nq, w, generator=g) * 4 - 2)).to(torch.bfloat16).cuda()
    v = ((torch.rand(batch, nq, w, generator=g) * 2 - 1)).to(torch.bfloat16).cuda()
    o1 = torch.full((batch, nq, w), float("nan"), dtype=torch.bfloat16, device="cuda")
    o2 = torch.full_like(o1, float("nan"))
    dit._ck(E.lib().exn_test_attention(dit.h, q.data_ptr(), k.data_ptr(), v.data_ptr(), o1.data_ptr(),
                                       batch, nq, q0, p, nq, 8, 264, heads, nq))
    ms = ctypes.c_double(-1.0)
    dit._ck(E.lib().exn_test_attention_timed(dit.h, q.data_ptr(), k.data_ptr(), v.data_ptr(), o2.data_ptr(),
                                             batch, nq, q0, p, nq, 8, 264, heads, nq, 5, ctypes.byref(ms)))
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
    assert ms.value > 0


# (kind, m, in, out, act, piece): the DiT's four GEMV calls (timestep MLP 256 -> W and W -> W with
# SiLU, the modulation W -> 4W with tanh on its gate pieces, norm_out) plus bf16 / f32 weights and a
# row count that is not a multiple of a warp's rows
GEMV_CASES = [
    (0, 2, 256, 4096, 1, 0),
    (0, 2, 4096, 4096, 1, 0),
    (0, 2, 4096, 16384, 2, 4096),
    (0, 1, 4096, 4096, 0, 0),
    (0, 1, 4096, 1000, 0, 0),
    (1, 2, 4096, 1024, 1, 0),
    (2, 2, 4096, 1024, 2, 256),
]


@pytest.mark.parametrize("case", GEMV_CASES, ids=["kind%d-m%d-%dx%d-act%d" % c[:5] for c in GEMV_CASES])
def test_gemv_matches_numpy(dit, case):
    """k_gemv (the timestep MLP and modulation, src/cuda-dit.lisp:157-167) against a float64 product of
    the same weights: Q8_0 values q * d exactly as upload-dit keeps them, bf16 or f32 matrices.  The
    kernel accumulates in fp32 over up to 4096 terms, so the bound is 2e-5 of the output's scale."""
    import ctypes
    kind, m, k_in, n_out, act, piece = case
    rs = np.random.default_rng(k_in + n_out + kind)
    x = rs.standard_normal((m, k_in)).astype(np.float32)
    if kind == 0:
        q = rs.integers(-127, 128, (n_out, k_in)).astype(np.int8)
        dsc = (rs.uniform(0.5, 1.5, (n_out, k_in // 32)) * 0.02 / 127).astype(np.float16)
        w = q.astype(np.float64) * np.repeat(dsc.astype(np.float64), 32, axis=1)
        wd, dd = torch.from_numpy(q).cuda(), torch.from_numpy(dsc).cuda()
    elif kind == 1:
        wt = (torch.from_numpy(rs.standard_normal((n_out, k_in)).astype(np.float32)) * 0.02).to(torch.bfloat16)
        w = wt.double().numpy()
        wd, dd = wt.cuda(), None
    else:
        wf = (rs.standard_normal((n_out, k_in)) * 0.02).astype(np.float32)
        w = wf.astype(np.float64)
        wd, dd = torch.from_numpy(wf).cuda(), None
    want = x.astype(np.float64) @ w.T
    if act == 1:
        want = want / (1 + np.exp(-want))
    elif act == 2:
        pc = np.arange(n_out) // piece
        gate = (pc == 1) | (pc == 3)
        want[:, gate] = np.tanh(want[:, gate])
    xd = torch.from_numpy(x).cuda()
    y = torch.full((m, n_out), float("nan"), dtype=torch.float32, device="cuda")
    ms = ctypes.c_double(-1.0)
    dit._ck(E.lib().exn_test_gemv(dit.h, kind, wd.data_ptr(), dd.data_ptr() if dd is not None else None,
                                  xd.data_ptr(), y.data_ptr(), m, k_in, n_out, act, piece, 10, ctypes.byref(ms)))
    got = y.cpu().numpy().astype(np.float64)
    err = np.abs(got - want).max() / np.abs(want).max()
    wbytes = n_out * k_in * (1.0625 if kind == 0 else (2 if kind == 1 else 4))
    print("\nGEMV kind %d, %d x %d -> %d: max err %.2e of the output's scale; %.1f us a launch, %.2f TB/s of "
          "weights (10 launches back to back: weights that fit stay in L2)"
          % (kind, m, k_in, n_out, err, ms.value * 1e3, wbytes / (ms.value * 1e-3) / 1e12))
    assert np.isfinite(got).all() and err < 2e-5


def test_ln_mod_row_selection(dit):
    # metal-kernels-test.lisp:91-102: rows n0 + t < p take the second modulation row
    wd, n, n0, p = 4096, 9, 3, 6
    rs = np.random.default_rng(7)
    x = (rs.uniform(-1, 1, (n, wd)) * 50).astype(np.float32)
    mod = rs.uniform(-1, 1, (2, wd)).astype(np.float32)
    xd, md = torch.from_numpy(x).cuda(), torch.from_numpy(mod).cuda()
    y = torch.empty(n, wd, dtype=torch.bfloat16, device="cuda")
    dit._ck(E.lib().exn_test_ln_mod(dit.h, xd.data_ptr(), y.data_ptr(), md.data_ptr(), n, wd, n0, p))
    xx = x.astype(np.float64)
    m = xx.mean(1, keepdims=True)
    inv = 1 / np.sqrt(((xx - m) ** 2).mean(1, keepdims=True) + 1e-6)
    row = np.where(n0 + np.arange(n) < p, 1, 0)
    want = (xx - m) * inv * (1 + mod[row].astype(np.float64))
    got = y.float().cpu().numpy()
    maxrel = np.abs(got - want).max() / np.abs(want).max()
    assert maxrel < 2 ** -8, maxrel   # bf16 output (it feeds a bf16 GEMM)
    exact = (got == torch.from_numpy(want).to(torch.bfloat16).float().numpy()).mean()
    assert exact > 0.99, exact


def test_synthetic_weights_match_the_oracle(dit):
    sw = O.SynthWeights.make(O.Shape(**TINY), seed=1)
    for name, dims in O.expected_tensors(O.Shape(**TINY)):
        if len(dims) != 2:
            continue
        want = bf16(sw(name)).view(torch.int16).numpy()
        got = np.empty(want.shape, dtype=np.int16)
        dit._ck(E.lib().exn_test_weight_bf16(dit.h, name.encode(), got.ctypes.data, got.size))
        assert np.array_equal(got, want), name


def test_qkv_epilogue_norm_rope(dit):
    # the fused to_q/to_k/to_v GEMM epilogue against ref_dit.py:135-139's arithmetic
    sh = O.Shape(**TINY)
    sw = O.SynthWeights.make(sh, seed=1)
    p, hh, ww = 5, 3, 4
    n0, n = 0, p + hh * ww
    rs = np.random.default_rng(3)
    y = bf16(rs.standard_normal((n, sh.width)))
    yd = y.cuda()
    q = torch.empty(n, sh.width, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(n + 3, sh.width, dtype=torch.bfloat16, device="cuda")
    v = torch.zeros(n + 3, sh.width, dtype=torch.bfloat16, device="cuda")
    dit._ck(E.lib().exn_test_qkv(dit.h, 1, yd.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), n, n0, p, hh, ww,
                                 n + 3))
    b = "transformer_blocks.1."
    yy = y.double().numpy()
    cos, sin = O.rope_tables(O.dit_positions(p, hh, ww))
    heads = sh.heads
    for name, out, norm in [("to_q", q, "norm_q"), ("to_k", k[:n], "norm_k"), ("to_v", v[:n], None)]:
        wq = bf16(sw(b + "attn." + name + ".weight")).double().numpy()
        want = (yy @ wq.T).reshape(n, heads, 128)
        if norm:
            want = O.rope(O.rmsnorm(want, sw.vec[b + "attn." + norm + ".weight"].astype(np.float64)), cos, sin)
        want = want.reshape(n, sh.width)
        got = out.float().cpu().numpy()
        maxrel = np.abs(got - want).max() / np.abs(want).max()
        assert maxrel < 2 ** -7, (name, maxrel)


def test_a_wait_that_runs_out_ends_in_a_timeout_status(dit):
    # failure detection without a GPU fault: a CTA waits, through the kernels' own bounded
    # mbarrier wait, on a barrier nothing arrives on (limit 50 ms); the call returns EXN_ETIMEOUT
    # with the kernels' message, and the handle works afterwards
    import time
    t0 = time.perf_counter()
    rc = E.lib().exn_test_wait_probe(dit.h, 0.05)
    dt = time.perf_counter() - t0
    assert rc == 6, rc                                  # EXN_ETIMEOUT
    assert b"gave up waiting" in E.lib().exn_last_error(dit.h)
    assert 0.04 < dt < 10.0, dt
    g = torch.Generator().manual_seed(5)
    a = torch.randn(128, 256, generator=g).to(torch.bfloat16).cuda()
    b = (torch.randn(256, 256, generator=g) * 0.05).to(torch.bfloat16).cuda()
    c = torch.full((128, 256), float("nan"), dtype=torch.float32, device="cuda")
    dit._ck(E.lib().exn_test_gemm(dit.h, a.data_ptr(), b.data_ptr(), c.data_ptr(), 128, 256, 256))
    ref = a.double() @ b.double().T
    assert (c.double() - ref).abs().max().item() / ref.abs().max().item() < 1e-5
