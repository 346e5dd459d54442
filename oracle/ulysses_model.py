"""A numpy model of the sequence-parallel (Ulysses) pass of libexn_b200.
TEST INFRASTRUCTURE ONLY: it runs one rank's share with the same sharding
rules as the library's run_step_sp (ex-nihilo_b200/csrc/dit.cpp) so the
tests can check the partitioning on CPU ranks (gloo) against the unsharded
oracle forward (oracle/dit_oracle.py, restating inspect/ref_dit.py).

Rank r of G holds prefix rows [r P/G, (r+1) P/G) on the first pass and image
rows [r N/G, (r+1) N/G); before attention an all-to-all trades its rows of
head group s for rank s's rows of its own head group r; after attention the
reverse.  ALL_TO_ALL(list of G arrays) -> list of G arrays (from each rank).
"""
from __future__ import annotations

import numpy as np

from . import dit_oracle as O


def forward_rank(wt, sh: O.Shape, ctx, latent, sigma, rank, world, all_to_all, ref=None):
    """This rank's columns [r N/G, (r+1) N/G) of the velocity (64 x N/G)."""
    G, r = world, rank
    W, HD = sh.width, sh.head_dim
    heads = sh.heads
    hg = heads // G
    ptext = ctx.shape[0]
    c, h, w = latent.shape
    N = h * w
    _, (scale1, gate1, scale2, gate2), sc = O.modulation(wt, sh, sigma)
    txt = O.rmsnorm(ctx, 1.0 + wt("txt_in.text_norm.weight"))
    txt = O.linear(O.gelu_tanh(O.linear(txt, wt("txt_in.in_layer.weight"))), wt("txt_in.out_layer.weight"))
    if ref is None:
        xp, P, b0, b1, refpos = txt, ptext, 0, 0, None
    else:
        a, rlat = ref
        rc, rh, rw = rlat.shape
        rimg = O.linear(rlat.reshape(rc, rh * rw).T, wt("img_in.weight"))
        xp = np.concatenate([txt[:a], rimg, txt[a:]])
        P, b0, b1, refpos = ptext + rh * rw, a, a + rh * rw, (a, rh, rw)
    assert P % G == 0 and N % G == 0 and heads % G == 0
    pl, Nl = P // G, N // G
    L = P + N
    img_all = O.linear(latent.reshape(c, N).T, wt("img_in.weight"))
    x = np.concatenate([xp[r * pl:(r + 1) * pl], img_all[r * Nl:(r + 1) * Nl]]).astype(np.float32)
    n_loc = pl + Nl
    rows = np.concatenate([np.arange(r * pl, (r + 1) * pl), P + np.arange(r * Nl, (r + 1) * Nl)])
    kind = np.where(np.arange(n_loc) < pl, 1, 0)               # prompt rows take modulation row 1
    cos_all, sin_all = O.rope_tables(O.dit_positions(P, h, w, refpos))
    cos, sin = cos_all[rows], sin_all[rows]
    order = np.concatenate([s * pl + np.arange(pl) for s in range(G)] + [P + s * Nl + np.arange(Nl) for s in range(G)])
    for il in range(sh.layers):
        b = "transformer_blocks.%d." % il
        y = O.layernorm(x) * (1.0 + scale1[kind])
        q = O.linear(y, wt(b + "attn.to_q.weight")).reshape(n_loc, heads, HD)
        k = O.linear(y, wt(b + "attn.to_k.weight")).reshape(n_loc, heads, HD)
        v = O.linear(y, wt(b + "attn.to_v.weight")).reshape(n_loc, heads, HD)
        q = O.rope(O.rmsnorm(q, wt(b + "attn.norm_q.weight")), cos, sin)
        k = O.rope(O.rmsnorm(k, wt(b + "attn.norm_k.weight")), cos, sin)
        packed = np.concatenate([q, k, v], axis=2)              # n_loc x heads x 3*HD
        got = all_to_all([np.ascontiguousarray(packed[:, s * hg:(s + 1) * hg]) for s in range(G)])
        # every rank's rows of my head group, back in sequence order
        pre = np.concatenate([g[:pl] for g in got])
        img = np.concatenate([g[pl:] for g in got])
        full = np.empty((L, hg, 3 * HD), dtype=np.float32)
        full[order] = np.concatenate([pre, img])
        qf, kf, vf = full[..., :HD], full[..., HD:2 * HD], full[..., 2 * HD:]
        att = O.attention(qf, kf, vf, 0, P, L, b0, b1)            # L x hg x HD
        back = all_to_all([np.ascontiguousarray(np.concatenate([att[s * pl:(s + 1) * pl],
                                                               att[P + s * Nl:P + (s + 1) * Nl]]))
                           for s in range(G)])
        att_loc = np.concatenate(back, axis=1).reshape(n_loc, W)   # head groups back into columns
        x = x + np.tanh(gate1[kind]) * O.linear(att_loc, wt(b + "attn.to_out.0.weight"))
        y = O.layernorm(x) * (1.0 + scale2[kind])
        gu = O.linear(y, wt(b + "img_mlp.gate_up.weight"))
        y = O.silu(gu[:, :sh.ffn]) * gu[:, sh.ffn:]
        x = (x + np.tanh(gate2[kind]) * O.linear(y, wt(b + "img_mlp.out.weight"))).astype(np.float32)
    xi = O.layernorm(x[pl:]) * (1.0 + sc)
    v = O.linear(xi, wt("proj_out.weight"))
    return v.T.astype(np.float32)                               # 64 x N/G
