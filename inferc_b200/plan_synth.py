"""Seeded synthetic *models* as optimized inferc plans (ONNX bytes).

There is no network for HuggingFace checkpoints, so these builders write the
plans that `inferc optimize` would produce for the two benchmark
architectures, with the weights of inferc_b200.synth:

  distilbert_plan  - the DistilBERT-architecture classifier after the fusion
                     passes (src/cli/main.cpp:270-277): FusedQKV,
                     FusedAttention (mask input = Unsqueeze(Equal(mask, 0)),
                     i.e. the [B,1,1,S] bool mask before Expand,
                     recognize_attention.cc:76-92), FusedLayerNorm,
                     FusedMatMulAddGELU, the out-projection and FFN2 left as
                     MatMul -> Add(bias) -> Add(residual), the position ids built
                     from Shape / Gather / Range, and the Gather(CLS) ->
                     Gemm(transB) -> Relu -> Gemm(transB) head.
  gpt2_plans       - the GPT-2 prefill ("no past") and single-token ("with
                     past") graphs that `inferc decode` runs
                     (src/cli/main.cpp:700-945): Gemm Conv1D projections
                     (transB=0), Split / Reshape / Transpose heads, Concat of
                     past_key_values.{i}.key/value into present.{i}.*, the
                     causal mask sliced from a lower-triangular bool buffer and
                     applied with Where(mask, scores, float32 min), Softmax,
                     GeluTanh, and the tied LM head MatMul(x, Transpose(wte)).

Node order and arithmetic follow the reference kernels' replay in
oracle/ref_capi.cc, so the reference's outputs (tests/golden/) pin them.
"""
from __future__ import annotations

import numpy as np

from . import onnx_io as ox
from .synth import EncoderConfig, Gpt2Config

FLOAT_MIN = float(np.finfo(np.float32).min)


def distilbert_plan(cfg: EncoderConfig, w: dict) -> bytes:
    g = ox.GraphBuilder("distilbert_optimized")
    H = cfg.hidden
    ids = g.input("input_ids", ox.INT64, ["batch", "seq"])
    mask = g.input("attention_mask", ox.INT64, ["batch", "seq"])
    for k, v in w.items():
        g.init(k, v)
    # position ids = Range(0, seq) from the ids' shape
    seq = g.one("Gather", [g.one("Shape", [ids]), g.const_i64(1)], axis=0)
    pos = g.one("Unsqueeze", [g.one("Range", [g.const_i64(0), seq, g.const_i64(1)]),
                              g.const_i64([0])])
    x = g.one("Add", [g.one("Gather", ["word_emb", ids], axis=0),
                      g.one("Gather", ["pos_emb", pos], axis=0)])
    x = g.one("FusedLayerNorm", [x, "emb_ln_g", "emb_ln_b"], domain="inferc",
              epsilon=float(cfg.ln_eps))
    # padding mask: true = masked, [B, 1, 1, S]
    cond = g.one("Unsqueeze", [g.one("Equal", [mask, g.const_i64(0)]), g.const_i64([1, 2])])
    for l in range(cfg.layers):
        q, k, v = g.add("FusedQKV", [x, f"wq.{l}", f"bq.{l}", f"wk.{l}", f"bk.{l}", f"wv.{l}",
                                      f"bv.{l}"], 3, domain="inferc")
        ctx = g.one("FusedAttention", [q, k, v, cond], domain="inferc", head_dim=H // cfg.heads,
                    fill=float(cfg.attn_fill))
        sa = g.one("Add", [g.one("Add", [g.one("MatMul", [ctx, f"wo.{l}"]), f"bo.{l}"]), x])
        x = g.one("FusedLayerNorm", [sa, f"ln1_g.{l}", f"ln1_b.{l}"], domain="inferc",
                  epsilon=float(cfg.ln_eps))
        hf = g.one("FusedMatMulAddGELU", [x, f"w1.{l}", f"b1.{l}"], domain="inferc")
        ff = g.one("Add", [g.one("Add", [g.one("MatMul", [hf, f"w2.{l}"]), f"b2.{l}"]), x])
        x = g.one("FusedLayerNorm", [ff, f"ln2_g.{l}", f"ln2_b.{l}"], domain="inferc",
                  epsilon=float(cfg.ln_eps))
    cls = g.one("Gather", [x, g.const_i64(0)], axis=1)
    pre = g.one("Relu", [g.one("Gemm", [cls, "pre_w", "pre_b"], transB=1)])
    g.add("Gemm", [pre, "cls_w", "cls_b"], outputs=["logits"], transB=1)
    g.output("logits", ox.FLOAT, ["batch", cfg.n_classes])
    return g.model()


def _gpt2_graph(cfg: Gpt2Config, w: dict, with_past: bool) -> bytes:
    g = ox.GraphBuilder("gpt2_with_past" if with_past else "gpt2")
    H, nH = cfg.hidden, cfg.heads
    hd = H // nH
    ids = g.input("input_ids", ox.INT64, [1, "seq"])
    g.input("attention_mask", ox.INT64, [1, "total"])
    past = []
    if with_past:
        for l in range(cfg.layers):
            past.append((g.input(f"past_key_values.{l}.key", ox.FLOAT, [1, nH, "past", hd]),
                         g.input(f"past_key_values.{l}.value", ox.FLOAT, [1, nH, "past", hd])))
    for k, v in w.items():
        g.init(k, v)
    causal = g.init("causal_bias",
                    np.tril(np.ones((cfg.max_pos, cfg.max_pos), bool)).reshape(
                        1, 1, cfg.max_pos, cfg.max_pos))
    n = g.one("Gather", [g.one("Shape", [ids]), g.const_i64(1)], axis=0)
    if with_past:
        past_len = g.one("Gather", [g.one("Shape", [past[0][0]]), g.const_i64(2)], axis=0)
    else:
        past_len = g.const_i64(0)
    total = g.one("Add", [past_len, n])
    pos = g.one("Unsqueeze", [g.one("Range", [past_len, total, g.const_i64(1)]),
                              g.const_i64([0])])
    x = g.one("Add", [g.one("Gather", ["wte", ids], axis=0), g.one("Gather", ["wpe", pos],
                                                                       axis=0)])
    # causal rows [past, total) and columns [0, total) of the lower-triangular buffer
    starts = g.one("Concat", [g.one("Unsqueeze", [past_len, g.const_i64([0])]),
                              g.const_i64([0])], axis=0)
    ends = g.one("Concat", [g.one("Unsqueeze", [total, g.const_i64([0])]),
                            g.one("Unsqueeze", [total, g.const_i64([0])])], axis=0)
    mask = g.one("Slice", [causal, starts, ends, g.const_i64([2, 3])])
    fill = g.const_f32(FLOAT_MIN)
    eight = g.const_f32(float(np.sqrt(np.float32(hd))))
    presents = []
    for l in range(cfg.layers):
        h = g.one("FusedLayerNorm", [x, f"ln1_g.{l}", f"ln1_b.{l}"], domain="inferc",
                  epsilon=float(cfg.ln_eps))
        qkv = g.one("Gemm", [g.one("Reshape", [h, g.const_i64([-1, H])]), f"attn_w.{l}",
                             f"attn_b.{l}"])
        q, k, v = g.add("Split", [g.one("Reshape", [qkv, g.const_i64([1, -1, 3 * H])]),
                                  g.const_i64([H, H, H])], 3, axis=2)

        def heads(t):
            return g.one("Transpose", [g.one("Reshape", [t, g.const_i64([1, -1, nH, hd])])],
                         perm=[0, 2, 1, 3])
        q, k, v = heads(q), heads(k), heads(v)
        kn, vn = f"present.{l}.key", f"present.{l}.value"
        if with_past:
            g.add("Concat", [past[l][0], k], outputs=[kn], axis=2)
            g.add("Concat", [past[l][1], v], outputs=[vn], axis=2)
        else:
            g.add("Identity", [k], outputs=[kn])
            g.add("Identity", [v], outputs=[vn])
        presents += [kn, vn]
        s = g.one("Div", [g.one("MatMul", [q, g.one("Transpose", [kn], perm=[0, 1, 3, 2])]),
                          eight])
        s = g.one("Where", [mask, s, fill])
        p = g.one("Softmax", [s], axis=-1)
        ctx = g.one("Reshape", [g.one("Transpose", [g.one("MatMul", [p, vn])], perm=[0, 2, 1, 3]),
                                g.const_i64([-1, H])])
        a = g.one("Gemm", [ctx, f"proj_w.{l}", f"proj_b.{l}"])
        x = g.one("Add", [g.one("Reshape", [a, g.const_i64([1, -1, H])]), x])
        h = g.one("FusedLayerNorm", [x, f"ln2_g.{l}", f"ln2_b.{l}"], domain="inferc",
                  epsilon=float(cfg.ln_eps))
        f = g.one("Gemm", [g.one("Reshape", [h, g.const_i64([-1, H])]), f"fc_w.{l}",
                           f"fc_b.{l}"])
        f = g.one("GeluTanh", [f], domain="inferc")
        m = g.one("Gemm", [f, f"fcproj_w.{l}", f"fcproj_b.{l}"])
        x = g.one("Add", [x, g.one("Reshape", [m, g.const_i64([1, -1, H])])])
    x = g.one("FusedLayerNorm", [x, "lnf_g", "lnf_b"], domain="inferc",
              epsilon=float(cfg.ln_eps))
    g.add("MatMul", [x, g.one("Transpose", ["wte"], perm=[1, 0])], outputs=["logits"])
    g.output("logits", ox.FLOAT, [1, "seq", cfg.vocab])
    for i, name in enumerate(presents):
        g.output(name, ox.FLOAT, [1, nH, "total", hd])
    return g.model()


def gpt2_plans(cfg: Gpt2Config, w: dict) -> tuple[bytes, bytes]:
    """(prefill graph, with-past graph) as `inferc decode --model / --past-model`."""
    return _gpt2_graph(cfg, w, False), _gpt2_graph(cfg, w, True)
