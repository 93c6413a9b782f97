"""The device executor on optimized ONNX plans, against the reference:

  - the DistilBERT-architecture plan (small config, config 0, the batch-8
    variable-length case and the full batch-256 bench workload) gives logits
    within 1e-4 of the reference kernels' (tests/golden/);
  - GPT-2 prefill + with-past plans decoded by the `inferc decode` loop give
    bit-identical greedy tokens (small config and the full 32 + 128 workload);
  - every glue op on small graphs against numpy restatements of the
    reference kernels (src/kernels/elementwise.cc, movement.cc, embedding.cc,
    activation.cc), including broadcasting, negative Slice steps, non-last
    Softmax / ReduceMean axes and the Gather range error.
"""
import os

import numpy as np
import pytest

from inferc_b200 import executor, onnx_io, plan_synth, synth
from inferc_b200.lib import InfercError
from tests.golden import make_golden

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LOGIT_TOL = 1e-4


def _enc(cfg, seed, ids, mask):
    g = executor.Graph(plan_synth.distilbert_plan(cfg, synth.encoder_weights(cfg, seed=seed)))
    return g.run_host({"input_ids": ids, "attention_mask": mask}, ["logits"])["logits"], g


def test_distilbert_plan_small_config():
    e = np.load(os.path.join(GOLD, "encoder.npz"))
    got, _ = _enc(synth.EncoderConfig(**make_golden.SMALL_ENC), 5, e["small_ids"], e["small_mask"])
    np.testing.assert_allclose(got, e["small_logits"], atol=LOGIT_TOL, rtol=0)


def test_distilbert_plan_full_config_c0_c4_and_rerun():
    e = np.load(os.path.join(GOLD, "encoder.npz"))
    cfg = synth.EncoderConfig()
    g = executor.Graph(plan_synth.distilbert_plan(cfg, synth.encoder_weights(cfg, seed=0)))
    for _ in range(2):  # a second run reuses the executor and its cached weights
        got = g.run_host({"input_ids": e["c0_ids"], "attention_mask": e["c0_mask"]},
                         ["logits"])["logits"]
        np.testing.assert_allclose(got, e["c0_logits"], atol=LOGIT_TOL, rtol=0)
        got = g.run_host({"input_ids": e["c4_ids"], "attention_mask": e["c4_mask"]},
                         ["logits"])["logits"]
        np.testing.assert_allclose(got, e["c4_logits"], atol=LOGIT_TOL, rtol=0)
    gold = np.load(os.path.join(GOLD, "encoder_c4_bench.npz"))
    ids, mask = synth.encoder_inputs(256, 128, seed=int(gold["seed"]), variable_lengths=True)
    got = g.run_host({"input_ids": ids, "attention_mask": mask}, ["logits"])["logits"]
    np.testing.assert_allclose(got, gold["logits"], atol=LOGIT_TOL, rtol=0)
    bad = e["c0_ids"].copy()
    bad[0, 3] = 10 ** 7
    with pytest.raises(InfercError, match="RANGE"):
        g.run_host({"input_ids": bad, "attention_mask": e["c0_mask"]}, ["logits"])
    got = g.run_host({"input_ids": e["c0_ids"], "attention_mask": e["c0_mask"]},
                     ["logits"])["logits"]
    np.testing.assert_allclose(got, e["c0_logits"], atol=LOGIT_TOL, rtol=0)


def test_distilbert_plan_fp16_range_rerun():
    """Activations beyond fp16's range (embedding LayerNorm gamma 1e5): the
    executor's split-fp16 planes raise the range flag and the run is redone
    on the fp32 operands; the logits still match the reference."""
    from inferc_b200 import structs
    from oracle import oracle
    cfg = synth.EncoderConfig(**make_golden.SMALL_ENC)
    w = synth.encoder_weights(cfg, seed=9)
    w["emb_ln_g"] = np.full_like(w["emb_ln_g"], 1e5)
    ids, mask = synth.encoder_inputs(3, 32, seed=4, vocab=cfg.vocab, variable_lengths=True)
    ref = oracle.port().encoder_forward(structs.encoder_struct(cfg, w), ids, mask, 2)
    g = executor.Graph(plan_synth.distilbert_plan(cfg, w))
    for _ in range(2):
        got = g.run_host({"input_ids": ids, "attention_mask": mask}, ["logits"])["logits"]
        np.testing.assert_allclose(got, ref, atol=LOGIT_TOL, rtol=1e-4)


@pytest.mark.parametrize("full", [False, True], ids=["small", "gpt2-small"])
def test_gpt2_plans_decode_tokens(full):
    d = np.load(os.path.join(GOLD, "decode.npz"))
    if full:
        cfg, seed, prompt, want = synth.Gpt2Config(), 0, d["c1_prompt"], d["c1_tokens"]
    else:
        cfg = synth.Gpt2Config(**make_golden.SMALL_GPT2)
        seed, prompt, want = 8, d["small_prompt"], d["small_tokens"]
    a, b = plan_synth.gpt2_plans(cfg, synth.gpt2_weights(cfg, seed=seed))
    pre, step = executor.Graph(a), executor.Graph(b)
    toks, ms = executor.greedy_decode(pre, step, cfg.layers, prompt, len(want))
    np.testing.assert_array_equal(toks, want)
    assert ms > 0


# ------------------------------------------------------------ glue ops

def _run(build, inputs, outs=("y",)):
    g = onnx_io.GraphBuilder("t")
    for k, v in inputs.items():
        code = {np.dtype(np.float32): 1, np.dtype(np.int64): 7, np.dtype(np.int32): 6,
                np.dtype(np.bool_): 9}[v.dtype]
        g.input(k, code, list(v.shape))
    build(g)
    for o in outs:
        g.output(o, 1, [])
    return executor.Graph(g.model()).run_host(inputs, list(outs))


RNG = np.random.default_rng(0)


def _f(*s):
    return RNG.standard_normal(s).astype(np.float32)


@pytest.mark.parametrize("op,fn", [("Add", np.add), ("Sub", np.subtract), ("Mul", np.multiply),
                                   ("Div", np.divide)])
@pytest.mark.parametrize("sa,sb", [((4, 8, 16), (16,)), ((4, 8, 16), (4, 8, 16)),
                                   ((4, 1, 16), (1, 8, 1)), ((3,), ()), ((5, 7), (5, 1))])
def test_binary_broadcast(op, fn, sa, sb):
    a, b = _f(*sa), _f(*sb) + (3.0 if op == "Div" else 0.0)
    y = _run(lambda g: g.add(op, ["a", "b"], outputs=["y"]), {"a": a, "b": b})["y"]
    np.testing.assert_allclose(y, fn(a, b), rtol=1e-6, atol=1e-6)


def test_int64_arith_pow_and_equal_where_cast():
    a = np.array([[7, -3, 12]], np.int64)
    b = np.array([2, 2, 5], np.int64)
    r = _run(lambda g: (g.add("Div", ["a", "b"], outputs=["d"]),
                        g.add("Pow", ["a", "b"], outputs=["p"])), {"a": a, "b": b}, ("d", "p"))
    np.testing.assert_array_equal(r["d"], np.trunc(a / b).astype(np.int64))  # C++ '/'
    np.testing.assert_array_equal(r["p"], (a.astype(float) ** b).astype(np.int64))
    x, y0 = _f(2, 3, 5), _f(5)
    m = np.array([[1], [0], [3]], np.int64)

    def build(g):
        c = g.one("Equal", ["m", g.const_i64(0)])
        g.add("Where", [c, "x", "y0"], outputs=["w"])
        g.add("Cast", [c], outputs=["cf"], to=1)
        g.add("Cast", ["m"], outputs=["mf"], to=1)
    r = _run(build, {"m": m, "x": x, "y0": y0}, ("w", "cf", "mf"))
    np.testing.assert_array_equal(r["w"], np.where(m == 0, x, y0))
    np.testing.assert_array_equal(r["cf"], (m == 0).astype(np.float32))
    np.testing.assert_array_equal(r["mf"], m.astype(np.float32))


def test_unary_and_activations():
    x = _f(3, 50) * 3
    r = _run(lambda g: [g.add(o, ["x"], outputs=[o.lower()], **({"domain": "inferc"}
                                                              if o.startswith("Gelu") else {}))
                        for o in ("Sqrt", "Erf", "Relu", "Tanh", "Neg", "Abs", "Gelu",
                                  "GeluTanh")],
             {"x": x}, ("sqrt", "erf", "relu", "tanh", "neg", "abs", "gelu", "gelutanh"))
    from math import erf
    np.testing.assert_allclose(r["sqrt"], np.sqrt(x), rtol=1e-6, equal_nan=True)
    np.testing.assert_allclose(r["erf"], np.vectorize(erf)(x), atol=1e-6)
    np.testing.assert_array_equal(r["relu"], np.maximum(x, 0))
    np.testing.assert_allclose(r["tanh"], np.tanh(x), atol=1e-6)
    np.testing.assert_array_equal(r["neg"], -x)
    np.testing.assert_array_equal(r["abs"], np.abs(x))
    np.testing.assert_allclose(r["gelu"], 0.5 * x * (1 + np.vectorize(erf)(x / np.sqrt(2))),
                               atol=1e-5)
    gt = 0.5 * x * (1 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))
    np.testing.assert_allclose(r["gelutanh"], gt, atol=1e-5)


def test_movement_ops():
    x = _f(2, 3, 4, 5)

    def build(g):
        g.add("Transpose", ["x"], outputs=["t"], perm=[2, 0, 3, 1])
        g.add("Slice", ["x", g.const_i64([3, -1]), g.const_i64([0, -6]), g.const_i64([2, 3]),
                        g.const_i64([-1, -2])], outputs=["s"])
        g.add("Concat", ["x", "x"], outputs=["c"], axis=2)
        g.add("Expand", [g.one("Slice", ["x", g.const_i64([0]), g.const_i64([1]),
                                         g.const_i64([1])]), g.const_i64([2, 3, 4, 5])],
              outputs=["e"])
        p0, p1 = g.add("Split", ["x", g.const_i64([1, 4])], 2, axis=3)
        g.add("Identity", [p1], outputs=["sp"])
        g.add("Reshape", [g.one("Unsqueeze", [g.one("Squeeze", [g.one("Slice", [
            "x", g.const_i64([0]), g.const_i64([1]), g.const_i64([0])])], axes=[0]),
                                               g.const_i64([1])]), g.const_i64([3, -1])],
              outputs=["r"])
    r = _run(build, {"x": x}, ("t", "s", "c", "e", "sp", "r"))
    np.testing.assert_array_equal(r["t"], x.transpose(2, 0, 3, 1))
    # the reference clamps a negative end to 0 (movement.cc:219-224), unlike numpy
    np.testing.assert_array_equal(r["s"], x[:, :, 3:0:-1, 4:0:-2])
    np.testing.assert_array_equal(r["c"], np.concatenate([x, x], 2))
    np.testing.assert_array_equal(r["e"], np.broadcast_to(x[:, :1], x.shape))
    np.testing.assert_array_equal(r["sp"], x[..., 1:])
    np.testing.assert_array_equal(r["r"], x[0].reshape(3, -1))


def test_gather_softmax_reduce_matmul_gemm():
    x, w = _f(6, 5), _f(4, 6, 7)
    idx = np.array([[2, -1], [0, 5]], np.int64)
    a, b, c = _f(3, 2, 5, 4), _f(2, 4, 6), _f(6)

    def build(g):
        g.add("Gather", ["x", "idx"], outputs=["ga"], axis=0)
        g.add("Gather", ["w", "idx"], outputs=["gb"], axis=1)
        g.add("Softmax", ["w"], outputs=["sm"], axis=1)
        g.add("ReduceMean", ["w"], outputs=["rm"], axes=[0, 2], keepdims=1)
        g.add("MatMul", ["a", "b"], outputs=["mm"])
        g.add("Gemm", ["x", g.one("Transpose", ["x"], perm=[1, 0]), "c"], outputs=["gm"],
              alpha=0.5, beta=2.0)
    r = _run(build, {"x": x, "w": w, "idx": idx, "a": a, "b": b, "c": c},
             ("ga", "gb", "sm", "rm", "mm", "gm"))
    np.testing.assert_array_equal(r["ga"], x[idx])
    np.testing.assert_array_equal(r["gb"], w[:, idx % 6])
    e = np.exp(w - w.max(1, keepdims=True))
    np.testing.assert_allclose(r["sm"], e / e.sum(1, keepdims=True), atol=1e-6)
    np.testing.assert_allclose(r["rm"], w.mean(axis=(0, 2), keepdims=True), atol=1e-6)
    np.testing.assert_allclose(r["mm"], np.matmul(a, b), atol=1e-4)
    np.testing.assert_allclose(r["gm"], 0.5 * x @ x.T + 2.0 * c, atol=1e-4)


def test_shape_metadata_folds_and_range_constant_of_shape():
    x = _f(3, 7)

    def build(g):
        n = g.one("Gather", [g.one("Shape", ["x"]), g.const_i64(1)], axis=0)
        g.add("Cast", [g.one("Range", [g.const_i64(2), n, g.const_i64(2)])], outputs=["rg"],
              to=1)
        g.add("ConstantOfShape", [g.one("Shape", ["x"])], outputs=["z"],
              value=np.array([2.5], np.float32))
        g.add("Constant", [], outputs=["k"], value=np.array([[1, 2]], np.int64))
        g.add("Cast", ["k"], outputs=["kf"], to=1)
    r = _run(build, {"x": x}, ("rg", "z", "kf"))
    np.testing.assert_array_equal(r["rg"], np.arange(2, 7, 2, dtype=np.float32))
    np.testing.assert_array_equal(r["z"], np.full((3, 7), 2.5, np.float32))
    np.testing.assert_array_equal(r["kf"], np.array([[1, 2]], np.float32))


def test_errors_match_the_reference_messages():
    x = _f(2, 3)
    with pytest.raises(InfercError, match="RANGE"):
        _run(lambda g: g.add("Gather", ["x", g.const_i64([5])], outputs=["y"], axis=0),
             {"x": x})
    with pytest.raises(InfercError, match="missing tensor 'nope'"):
        _run(lambda g: g.add("Relu", ["nope"], outputs=["y"]), {"x": x})
    with pytest.raises(InfercError, match="broadcast mismatch"):
        _run(lambda g: g.add("Add", ["x", g.init("b", _f(4))], outputs=["y"]), {"x": x})
    with pytest.raises(InfercError, match="Cast: unsupported dtype pair"):
        _run(lambda g: g.add("Cast", ["x"], outputs=["y"], to=9), {"x": x})


def test_matmul_decode_shapes():
    """The with-past decode graph's MatMuls: one query row per head against a
    growing key block (batched, every matrix in one launch), and the tied LM
    head, a row vector by the folded Transpose of an initializer whose width
    is not a multiple of 4 (the row GEMV over the initializer itself)."""
    q, kt = _f(1, 12, 1, 64), _f(1, 12, 64, 161)
    p, v = _f(1, 12, 1, 161), _f(1, 12, 161, 64)
    x, wte = _f(1, 96), _f(1003, 96)

    def build(g):
        g.init("wte", wte)
        g.add("MatMul", ["q", "kt"], outputs=["s"])
        g.add("MatMul", ["p", "v"], outputs=["o"])
        g.add("MatMul", ["x", g.one("Transpose", ["wte"], perm=[1, 0])], outputs=["logits"])
    r = _run(build, {"q": q, "kt": kt, "p": p, "v": v, "x": x}, ("s", "o", "logits"))
    np.testing.assert_allclose(r["s"], np.matmul(q, kt), rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(r["o"], np.matmul(p, v), rtol=1e-5, atol=1e-4)
    np.testing.assert_allclose(r["logits"], x @ wte.T, rtol=1e-5, atol=1e-4)
