"""CPU tests of the oracle: the C restatement ("port") is pinned against
(a) the known-answer vectors of the reference's own tests
    (tests/kernels_test.cc, bench/amx/int4_gemv_amx.cc fixtures),
(b) golden fixtures produced by the reference's own kernel sources
    (tests/golden/*.npz, tests/golden/make_golden.py), and
(c) the reference build itself when oracle/_ref is present.
"""
import math
import os

import numpy as np
import pytest

from inferc_b200 import structs, synth
from oracle import oracle
from tests.golden import make_golden

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def port():
    return oracle.port()


# ---------------------------------------------------- (a) known answers


def test_attention_single_head_known_answer(port):
    # kernels_test.cc:222-236
    q = np.array([[[1, 0], [0, 1]]], np.float32)
    v = np.array([[[1, 2], [3, 4]]], np.float32)
    out = port.fused_attention(q, q.copy(), v, None, 2, -1e30)
    np.testing.assert_allclose(out.ravel(), [1.6604, 2.6604, 2.3396, 3.3396], atol=1e-3)


def test_attention_mask_zeros_out_key(port):
    # kernels_test.cc:238-253: mask [1,1,1,2] hides key 1 -> every row = V[0]
    q = np.array([[[1, 0], [0, 1]]], np.float32)
    v = np.array([[[1, 2], [3, 4]]], np.float32)
    mask = np.array([0, 1], np.uint8).reshape(1, 1, 1, 2)
    out = port.fused_attention(q, q.copy(), v, mask, 2, -1e30)
    np.testing.assert_allclose(out.ravel(), [1, 2, 1, 2], atol=1e-3)


def test_gelu_tanh_formula(port):
    # kernels_test.cc:255-265
    x = np.array([-1.0, 0.0, 2.0], np.float32)
    ref = [0.5 * v * (1 + math.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3))) for v in x]
    np.testing.assert_allclose(port.gelu_tanh(x), ref, atol=1e-5)


def test_gelu_known_values(port):
    # kernels_test.cc:304-311
    y = port.gelu(np.array([0.0, 1.0, -1.0], np.float32))
    np.testing.assert_allclose(y, [0.0, 0.8413447, -0.1586553], atol=1e-5)


def test_softmax_numerically_stable(port):
    # kernels_test.cc:313-327
    y = port.softmax(np.array([[1000, 1001, 999, 1002]], np.float32))
    assert np.isfinite(y).all()
    assert abs(y.sum() - 1) < 1e-5
    assert y[0, 3] > y[0, 2] and y[0, 3] > y[0, 1]


def test_layernorm_mean_zero_var_one(port):
    # kernels_test.cc:343-362
    x = np.array([[1, 2, 3, 4], [10, 20, 30, 40]], np.float32)
    y = port.layernorm(x, np.ones(4, np.float32), np.zeros(4, np.float32), 1e-5)
    assert np.abs(y.mean(1)).max() < 1e-4
    assert np.abs(y.var(1) - 1).max() < 5e-3


def test_gemm_known_answers(port):
    # kernels_test.cc:94-110 style: bias broadcast, alpha/beta, transB
    a = np.array([[1, 2], [3, 4]], np.float32)
    b = np.array([[5, 6], [7, 8]], np.float32)
    c = np.array([1, 1], np.float32)
    np.testing.assert_array_equal(port.gemm(a, b, c), [[20, 23], [44, 51]])
    np.testing.assert_array_equal(port.gemm(a, b, c, 2.0, 0.5, False, True),
                                  [[34.5, 46.5], [78.5, 106.5]])


def _int4_fixture():
    # int4_gemv_amx.cc:481-488, :533-540
    N, K = 16, 256
    w = np.array([(i * 31) & 0xFF for i in range(N * K // 2)], np.uint8).reshape(N, K // 2)
    x = np.sin(0.07 * np.arange(K)).astype(np.float32)
    scales = np.array([0.05 + 0.01 * (i % 7) for i in range(N)], np.float32)
    return w, x, scales


def _int4_exact(w, scales, x):
    """Independent restatement: nibble order, fp32 weight, float64 sum."""
    K = x.size
    q = np.empty((w.shape[0], K), np.int64)
    q[:, 0::2] = (w & 0xF).astype(np.int64) - 8
    q[:, 1::2] = (w >> 4).astype(np.int64) - 8
    wf = (scales[:, None] * q.astype(np.float32)).astype(np.float32)
    return (wf.astype(np.float64) * x.astype(np.float64)).sum(1).astype(np.float32)


def test_int4_rowscale_reference_fixture(port):
    w, x, scales = _int4_fixture()
    y = port.int4_gemv_rowscale(w, scales, x)
    np.testing.assert_allclose(y, _int4_exact(w, scales, x), rtol=0, atol=1e-6)
    yt = port.int4_gemv(w, 0.125, x)
    np.testing.assert_allclose(yt, _int4_exact(w, np.full(16, 0.125, np.float32), x), atol=1e-6)


def test_int4_pack_layout():
    q = np.array([[-8, 7, 0, -1]], np.int8)
    packed = synth.pack_int4(q)
    # byte0 = (q0+8) | (q1+8) << 4 = 0x0 | 0xF << 4; byte1 = 8 | 7 << 4
    assert packed.tolist() == [[0xF0, 0x78]]


def test_argmax_first_max_wins(port):
    assert port.argmax(np.array([1, 3, 3, 2], np.float32)) == 1
    assert port.argmax(np.array([5], np.float32)) == 0


# ---------------------------------------------------- (b) golden fixtures


def test_port_matches_reference_golden_ops(port):
    g = np.load(os.path.join(GOLD, "ops.npz"))
    i = make_golden.ops_inputs()
    np.testing.assert_allclose(port.layernorm(i["ln_x"], i["ln_g"], i["ln_b"], 1e-12), g["ln_y"],
                               atol=2e-6)
    np.testing.assert_allclose(port.fused_matmul_add_gelu(i["mmg_x"], i["mmg_w"], i["mmg_b"]),
                               g["mmg_y"], atol=2e-6)
    q, k, v = port.fused_qkv(i["mmg_x"], i["qkv_wq"], i["qkv_bq"], i["qkv_wk"], i["qkv_bk"],
                             i["qkv_wv"], i["qkv_bv"])
    for a, n in ((q, "qkv_q"), (k, "qkv_k"), (v, "qkv_v")):
        np.testing.assert_allclose(a, g[n], atol=2e-6)
    np.testing.assert_allclose(port.fused_attention(i["attn_q"], i["attn_k"], i["attn_v"],
                                                    i["attn_mask"], 64, -3.0e38),
                               g["attn_o"], atol=2e-6)
    np.testing.assert_allclose(port.gemm(i["gemm_a"], i["gemm_b"], i["gemm_c"], 0.5, 2.0,
                                         False, True), g["gemm_y"], atol=2e-5)
    np.testing.assert_allclose(port.gemm(i["gemv_a"], i["gemv_b"], i["gemv_c"]), g["gemv_y"],
                               atol=2e-6)
    np.testing.assert_allclose(port.gelu_tanh(i["gt_x"]), g["gt_y"], atol=1e-6)
    np.testing.assert_allclose(port.gelu(i["gt_x"]), g["ge_y"], atol=1e-6)
    np.testing.assert_allclose(port.softmax(i["sm_x"]), g["sm_y"], atol=1e-7)


def test_port_encoder_matches_reference_golden(port):
    g = np.load(os.path.join(GOLD, "encoder.npz"))
    cfg = synth.EncoderConfig(**make_golden.SMALL_ENC)
    w = synth.encoder_weights(cfg, seed=5)
    logits = port.encoder_forward(structs.encoder_struct(cfg, w), g["small_ids"], g["small_mask"],
                                  2)
    np.testing.assert_allclose(logits, g["small_logits"], atol=1e-5)


def test_port_matches_c4_bench_golden(port):
    """The bench workload's fixture (reference logits of all 256 sequences):
    the port agrees on a spread of sequences, so the fixture and the port pin
    each other."""
    g = np.load(os.path.join(GOLD, "encoder_c4_bench.npz"))
    assert g["logits"].shape == (256, 2)
    cfg = synth.EncoderConfig()
    ids, mask = synth.encoder_inputs(256, 128, seed=int(g["seed"]), variable_lengths=True)
    rows = [0, 97, 255]
    got = port.encoder_forward(structs.encoder_struct(cfg, synth.encoder_weights(cfg, seed=0)),
                               ids[rows], mask[rows], 2)
    np.testing.assert_allclose(got, g["logits"][rows], atol=1e-5)


def test_port_decode_matches_reference_golden(port):
    g = np.load(os.path.join(GOLD, "decode.npz"))
    cfg = synth.Gpt2Config(**make_golden.SMALL_GPT2)
    w = synth.gpt2_weights(cfg, seed=8)
    toks, _ = port.gpt2_decode(structs.gpt2_struct(cfg, w), g["small_prompt"],
                               len(g["small_tokens"]))
    np.testing.assert_array_equal(toks, g["small_tokens"])


def test_synth_is_deterministic():
    a = synth.encoder_inputs(4, 128, seed=7, variable_lengths=True)
    b = synth.encoder_inputs(4, 128, seed=7, variable_lengths=True)
    np.testing.assert_array_equal(a[0], b[0])
    ids, mask = a
    lens = mask.sum(1)
    assert (lens >= 16).all() and (lens <= 128).all()
    assert (ids[:, 0] == 101).all()
    for r in range(4):
        assert ids[r, lens[r] - 1] == 102 and (ids[r, lens[r]:] == 0).all()


# ---------------------------------------------------- (c) the reference build


@pytest.mark.skipif(oracle.ref() is None, reason="reference kernels not built here")
def test_port_matches_reference_build_random(port):
    ref = oracle.ref()
    rng = np.random.default_rng(3)
    q, k, v = [rng.standard_normal((2, 45, 192), dtype=np.float32) for _ in range(3)]
    m = (rng.random((2, 1, 45, 45)) < 0.2).astype(np.uint8)
    m[0, 0, 3, :] = 1  # a fully masked row -> uniform weights in both
    np.testing.assert_allclose(port.fused_attention(q, k, v, m, 64, -3.0e38),
                               ref.fused_attention(q, k, v, m, 64, -3.0e38), atol=2e-6)
    x = rng.standard_normal((19, 300), dtype=np.float32)
    gm = rng.standard_normal(300, dtype=np.float32)
    np.testing.assert_allclose(port.layernorm(x, gm, gm, 1e-5), ref.layernorm(x, gm, gm, 1e-5),
                               atol=2e-6)


def test_int4_round_trip_properties():
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((96, 40)) * 0.02).astype(np.float32)
    w[:, 3] = 0.0  # an all-zero output row gets scale 1
    m = synth.quantize_int4_rowscale(w)
    assert m.w.shape == (40, 48) and m.scales[3] == 1.0
    dq = synth.dequantize_int4_rowscale(m)
    assert dq.shape == w.shape
    s = np.abs(w).max(0) / np.float32(7)
    s[3] = 1
    assert (np.abs(dq - w) <= s / 2 + 1e-9).all()  # round to nearest
    wt = synth.dequantize_int4_rowscale(synth.quantize_int4_rowscale(w.T.copy(), trans=True),
                                        trans=True)
    np.testing.assert_array_equal(wt, dq.T)


def test_port_int4_decode_matches_reference_golden(port):
    g = np.load(os.path.join(GOLD, "decode_int4.npz"))
    cfg = synth.Gpt2Config(**make_golden.SMALL_GPT2)
    dq = synth.gpt2_weights_int4_dequantized(cfg, synth.gpt2_weights(cfg, seed=8))
    toks, _ = port.gpt2_decode_lm(structs.gpt2_struct(cfg, dq), dq["lm_head"], g["small_prompt"],
                                  len(g["small_tokens"]))
    np.testing.assert_array_equal(toks, g["small_tokens"])
