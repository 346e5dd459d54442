"""exn_qkv_noalloc: the fused QKV GEMM (RMSNorm + RoPE epilogue) for callers that cannot call
cudaMalloc, e.g. a host running the DiT on a GPU lent by another server whose allocator already
accounts for the device's memory.  Its RoPE scratch is a fixed device array of the library, not a
buffer grown at run time.

Checked through the C ABI against exn_test_qkv, which computes the same product with step
buffers it allocates: two calls of exn_qkv_noalloc in a row, with different sequence layouts (the
second reads table rows the first one wrote for other positions, so a row it failed to rewrite
would show), each equal to exn_test_qkv's output on the same inputs.  This file is collected last
so that a run stopping at its first failure has run every other test before it."""
import pytest

import exn_b200 as E

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TINY = dict(width=256, layers=2, ffn=768, context=256)
MAX_ROWS = 8704        # the rows of RoPE table the fixed scratch holds


@pytest.fixture(scope="module")
def dit():
    d = E.Dit(**TINY)
    d.load_synthetic(1)
    yield d
    d.close()


def _qkv(d, fn, layer, y, n, n0, p, hh, ww, kv_rows):
    w = d.cfg.width
    q = torch.full((n, w), float("nan"), dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(kv_rows, w, dtype=torch.bfloat16, device="cuda")
    v = torch.zeros(kv_rows, w, dtype=torch.bfloat16, device="cuda")
    d._ck(fn(d.h, layer, y.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), n, n0, p, hh, ww, kv_rows))
    torch.cuda.synchronize()
    return q.cpu(), k.cpu(), v.cpu()


def test_noalloc_qkv_equals_the_allocating_entry_point(dit):
    # (layer, n, n0, p, hh, ww): a first pass over a 9-row prompt and a 6 x 5 picture, then the
    # image rows only of a 5-row prompt and a 3 x 4 picture (their RoPE rows differ from the first's)
    cases = [(1, 39, 0, 9, 6, 5), (0, 12, 5, 5, 3, 4)]
    g = torch.Generator().manual_seed(17)
    ys = [torch.randn(n, dit.cfg.width, generator=g).to(torch.bfloat16).cuda() for _, n, *_ in cases]
    got = [_qkv(dit, E.lib().exn_qkv_noalloc, layer, y, n, n0, p, hh, ww, n0 + n + 3)
           for (layer, n, n0, p, hh, ww), y in zip(cases, ys)]
    want = [_qkv(dit, E.lib().exn_test_qkv, layer, y, n, n0, p, hh, ww, n0 + n + 3)
            for (layer, n, n0, p, hh, ww), y in zip(cases, ys)]
    for case, gq, wq in zip(cases, got, want):
        for name, a, b in zip("qkv", gq, wq):
            assert torch.isfinite(a.float()).all(), (case, name)
            # the same kernels on the same inputs: the same bits
            assert torch.equal(a.view(torch.int16), b.view(torch.int16)), (case, name)


def test_noalloc_qkv_rejects_a_sequence_beyond_its_scratch(dit):
    w = dit.cfg.width
    y = torch.zeros(1, w, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(2, w, dtype=torch.bfloat16, device="cuda")
    # p + hh x ww = 8705 rows, one more than the fixed table holds
    rc = E.lib().exn_qkv_noalloc(dit.h, 0, y.data_ptr(), out.data_ptr(), out.data_ptr(), out.data_ptr(), 1, 0,
                                 MAX_ROWS - 64 * 64 + 1, 64, 64, 2)
    assert rc == 1                                              # EXN_EINVAL
    msg = E.lib().exn_last_error(dit.h).decode()
    assert "8705" in msg and str(MAX_ROWS) in msg, msg
