"""Generate ``encoder_small.npz``: the prompt encoder's golden states from transformers' own
Qwen3-VL text model.

    python tests/golden/make_encoder_golden.py

The reference runs its prompt encoder (Qwen3-VL-8B's text model) through illatio, a sibling
project that is not in the reference tree, so the published implementation stands in for it:
``transformers.models.qwen3_vl.Qwen3VLTextModel`` (transformers 5.5 in this image), in float32
with eager attention, at a small shape (``oracle.encoder_oracle.SMALL``: width 512, 4 query and
2 key/value heads of 128, FFN 1024, 2 blocks, vocabulary 512, rope theta 5e6, M-RoPE sections
24/20/20 interleaved).  Its weights are the oracle's synthetic ones (Q8_0 matrices dequantised,
fp32 vectors).  What is stored, per case, is what ex-nihilo's ``encoder-states``
(src/encoder.lisp:143-183) reads: the last block's output, before the final norm, captured with
a forward hook on that block.

Cases: a text prompt (positions (i, i, i)) and an edit prompt's layout (6 text tokens, a 3 x 5
grid of picture pads at M-RoPE positions (a0, a0 + r, a0 + c), 9 text tokens after), as
src/encoder.lisp:116-123 builds its positions.  Only this script imports transformers; the tests
read the stored vectors.
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import encoder_oracle as E  # noqa: E402

CASES = {
    "text": dict(n=40, positions=None, seed=0),
    "edit": dict(n=30, positions=(6, 3, 5, 9), seed=1),
}


def hf_model(sh: E.EncShape, wt):
    import torch
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLTextConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

    cfg = Qwen3VLTextConfig(vocab_size=sh.vocab, hidden_size=sh.width, intermediate_size=sh.ffn,
                            num_hidden_layers=sh.layers, num_attention_heads=sh.heads,
                            num_key_value_heads=sh.kv_heads, head_dim=sh.head_dim, rms_norm_eps=sh.eps,
                            rope_parameters={"rope_type": "default", "rope_theta": sh.theta,
                                             "mrope_section": [24, 20, 20], "mrope_interleaved": True},
                            attention_bias=False)
    cfg._attn_implementation = "eager"
    m = Qwen3VLTextModel(cfg).float().eval()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))  # noqa: E731
    with torch.no_grad():
        m.embed_tokens.weight.copy_(t(wt("token_embd.weight")))
        for i, layer in enumerate(m.layers):
            b = "blk.%d." % i
            layer.input_layernorm.weight.copy_(t(wt(b + "attn_norm.weight")))
            layer.post_attention_layernorm.weight.copy_(t(wt(b + "ffn_norm.weight")))
            a = layer.self_attn
            a.q_proj.weight.copy_(t(wt(b + "attn_q.weight")))
            a.k_proj.weight.copy_(t(wt(b + "attn_k.weight")))
            a.v_proj.weight.copy_(t(wt(b + "attn_v.weight")))
            a.o_proj.weight.copy_(t(wt(b + "attn_output.weight")))
            a.q_norm.weight.copy_(t(wt(b + "attn_q_norm.weight")))
            a.k_norm.weight.copy_(t(wt(b + "attn_k_norm.weight")))
            layer.mlp.gate_proj.weight.copy_(t(wt(b + "ffn_gate.weight")))
            layer.mlp.up_proj.weight.copy_(t(wt(b + "ffn_up.weight")))
            layer.mlp.down_proj.weight.copy_(t(wt(b + "ffn_down.weight")))
    return m


def run_hf(m, ids, positions):
    import torch
    got = {}
    h = m.layers[-1].register_forward_hook(lambda mod, inp, out: got.__setitem__("x", out))
    try:
        pos = torch.from_numpy(positions.T.astype(np.int64))[:, None, :]   # (3, 1, n): t, h, w
        text = torch.arange(len(ids))[None, None, :]                         # the causal mask's positions
        with torch.no_grad():
            m(input_ids=torch.from_numpy(ids.astype(np.int64))[None], position_ids=torch.cat([text, pos], 0),
              use_cache=False)
    finally:
        h.remove()
    x = got["x"][0] if isinstance(got["x"], tuple) else got["x"]
    return x[0].float().numpy()


def main():
    import transformers
    sh = E.SMALL
    wt = E.SynthEncoder(sh, seed=1)
    m = hf_model(sh, wt)
    out = {"transformers_version": np.array(transformers.__version__)}
    for name, c in CASES.items():
        ids = E.synth_ids(sh, c["n"], seed=c["seed"])
        pos = E.text_positions(c["n"]) if c["positions"] is None else E.edit_positions(*c["positions"])
        assert len(pos) == c["n"]
        x = run_hf(m, ids, pos)
        mine = E.states(wt, sh, ids, pos)
        err = np.sqrt(((mine - x) ** 2).sum() / (x ** 2).sum())
        print("%s: n=%d |x| %.4g, oracle rel-L2 %.3g" % (name, c["n"], np.sqrt((x ** 2).mean()), err))
        out[name + "_ids"] = ids
        out[name + "_positions"] = pos
        out[name + "_states"] = x.astype(np.float32)
    dg = hashlib.sha256()
    for n, _ in E.encoder_tensors(sh):
        dg.update(np.ascontiguousarray(wt(n)).tobytes())
    out["weights_sha256"] = np.array(dg.hexdigest())
    np.savez_compressed(os.path.join(HERE, "encoder_small.npz"), **out)


if __name__ == "__main__":
    main()
