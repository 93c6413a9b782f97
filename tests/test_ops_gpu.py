"""GPU parity of every op entry point of libinferc_b200 against the CPU
oracle (C restatement, pinned to the reference) and the reference golden
fixtures. Each op runs through the C ABI (inferc_b200.ops -> ctypes)."""
import os

import numpy as np
import pytest
import torch

from inferc_b200 import ops, synth
from oracle import oracle
from tests.golden import make_golden

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def port():
    return oracle.port()


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(GOLD, "ops.npz")), make_golden.ops_inputs()


# ------------------------------------------------------------ LayerNorm

@pytest.mark.parametrize("rows,feat", [(1, 768), (33, 768), (128, 768), (5, 1024), (7, 100),
                                       (3, 4096), (0, 768)])
def test_layernorm(port, rows, feat):
    rng = np.random.default_rng(rows * 31 + feat)
    x = rng.standard_normal((rows, feat), dtype=np.float32) * 3 + 1
    g = rng.standard_normal(feat, dtype=np.float32)
    b = rng.standard_normal(feat, dtype=np.float32)
    y = host(ops.LayerNorm(T(x), T(g), T(b), 1e-5))
    if rows:
        np.testing.assert_allclose(y, port.layernorm(x, g, b, 1e-5), atol=1e-5, rtol=1e-5)


def test_layernorm_golden(gold):
    g, i = gold
    y = host(ops.LayerNorm(T(i["ln_x"]), T(i["ln_g"]), T(i["ln_b"]), 1e-12))
    np.testing.assert_allclose(y, g["ln_y"], atol=1e-5)


def test_layernorm_rejects_bad_shapes():
    x = torch.zeros(4, 8, device=DEV)
    with pytest.raises(RuntimeError):
        ops.LayerNorm(x, torch.ones(7, device=DEV), torch.zeros(7, device=DEV))
    with pytest.raises(RuntimeError):
        ops.LayerNorm(x.double(), torch.ones(8, device=DEV), torch.zeros(8, device=DEV))


# ------------------------------------------------------------ GEMM family

@pytest.mark.parametrize("M,K,N", [(1, 768, 3072), (17, 33, 50), (128, 768, 3072),
                                   (300, 768, 768), (64, 3072, 768), (0, 16, 16)])
def test_fused_matmul_add_gelu(port, M, K, N):
    rng = np.random.default_rng(M + K + N)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((K, N), dtype=np.float32) * 0.02).astype(np.float32)
    b = rng.standard_normal(N, dtype=np.float32) * 0.1
    y = host(ops.FusedMatMulAddGELU(T(x), T(w), T(b)))
    if M:
        ref = port.fused_matmul_add_gelu(x, w, b)
        # M >= 64 runs the tensor-core 3xTF32 kernel, whose fp32 accumulation
        # error grows with K (3e-5 of max |y| at K = 3072).
        np.testing.assert_allclose(y, ref, atol=2e-5 + 3e-5 * np.abs(ref).max(), rtol=1e-5)


def test_fused_matmul_add_gelu_golden_and_errors(gold):
    g, i = gold
    y = host(ops.FusedMatMulAddGELU(T(i["mmg_x"]), T(i["mmg_w"]), T(i["mmg_b"])))
    np.testing.assert_allclose(y, g["mmg_y"], atol=2e-5)
    with pytest.raises(RuntimeError, match="K mismatch"):
        ops.FusedMatMulAddGELU(torch.zeros(2, 5, device=DEV), torch.zeros(4, 3, device=DEV),
                               torch.zeros(3, device=DEV))


def test_fused_qkv_golden(gold):
    g, i = gold
    outs = ops.FusedQKVProjection(T(i["mmg_x"]), *[T(i["qkv_" + n]) for n in
                                                   ("wq", "bq", "wk", "bk", "wv", "bv")])
    for o, n in zip(outs, ("qkv_q", "qkv_k", "qkv_v")):
        np.testing.assert_allclose(host(o), g[n], atol=2e-5)


@pytest.mark.parametrize("ta,tb", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("clen", ["none", "row", "full", "scalar"])
def test_gemm_variants(port, ta, tb, clen):
    rng = np.random.default_rng(5)
    M, K, Nn = 37, 70, 45
    a = rng.standard_normal((K, M) if ta else (M, K), dtype=np.float32)
    b = rng.standard_normal((Nn, K) if tb else (K, Nn), dtype=np.float32)
    c = {"none": None, "row": rng.standard_normal(Nn, dtype=np.float32),
         "full": rng.standard_normal((M, Nn), dtype=np.float32),
         "scalar": np.array([0.75], np.float32)}[clen]
    y = host(ops.Gemm(T(a), T(b), None if c is None else T(c), 0.5, 2.0, ta, tb))
    ref = port.gemm(a, b, None if c is None else c.ravel(), 0.5, 2.0, ta, tb)
    np.testing.assert_allclose(y, ref, atol=1e-4, rtol=1e-5)


def test_gemm_m1_golden_and_bad_c(gold):
    g, i = gold
    y = host(ops.Gemm(T(i["gemv_a"]), T(i["gemv_b"]), T(i["gemv_c"])))
    np.testing.assert_allclose(y, g["gemv_y"], atol=1e-5)
    y = host(ops.Gemm(T(i["gemm_a"]), T(i["gemm_b"]), T(i["gemm_c"]), 0.5, 2.0, False, True))
    np.testing.assert_allclose(y, g["gemm_y"], atol=1e-4)
    with pytest.raises(RuntimeError, match="C shape"):
        ops.Gemm(torch.zeros(3, 4, device=DEV), torch.zeros(4, 5, device=DEV),
                 torch.zeros(4, device=DEV))


def test_matmul_matches_torch_fp64():
    rng = np.random.default_rng(9)
    a = rng.standard_normal((129, 257), dtype=np.float32)
    b = rng.standard_normal((257, 131), dtype=np.float32)
    y = host(ops.MatMul(T(a), T(b)))
    ref = a.astype(np.float64) @ b.astype(np.float64)
    np.testing.assert_allclose(y, ref, atol=1e-3, rtol=1e-5)


# ------------------------------------------------------------ attention

def _attn_case(B, S, H, hd, lens, seed):
    rng = np.random.default_rng(seed)
    q, k, v = [rng.standard_normal((B, S, H), dtype=np.float32) for _ in range(3)]
    mask = (np.arange(S)[None, :] >= np.asarray(lens)[:, None]).astype(np.uint8)
    return q, k, v, mask.reshape(B, 1, 1, S)


@pytest.mark.parametrize("B,S", [(1, 128), (8, 128), (2, 512), (3, 70), (1, 1), (2, 17)])
def test_fused_attention_padding_mask(port, B, S):
    lens = np.random.default_rng(B * S).integers(min(16, S), S + 1, size=B)
    q, k, v, m = _attn_case(B, S, 768, 64, lens, B + S)
    y = host(ops.FusedAttention(T(q), T(k), T(v), T(m), 64, -3.4028234663852886e38))
    np.testing.assert_allclose(y, port.fused_attention(q, k, v, m, 64, -3.4028234663852886e38),
                               atol=2e-5)


def test_fused_attention_golden(gold):
    g, i = gold
    y = host(ops.FusedAttention(T(i["attn_q"]), T(i["attn_k"]), T(i["attn_v"]),
                             T(i["attn_mask"]), 64, -3.0e38))
    np.testing.assert_allclose(y, g["attn_o"], atol=2e-5)


def test_fused_attention_known_answers():
    # kernels_test.cc:222-253 (head_dim 2: generic kernel)
    q = T(np.array([[[1, 0], [0, 1]]], np.float32))
    v = T(np.array([[[1, 2], [3, 4]]], np.float32))
    y = host(ops.FusedAttention(q, q.clone(), v, None, 2, -1e30)).ravel()
    np.testing.assert_allclose(y, [1.6604, 2.6604, 2.3396, 3.3396], atol=1e-3)
    m = T(np.array([0, 1], np.uint8).reshape(1, 1, 1, 2))
    y = host(ops.FusedAttention(q, q.clone(), v, m, 2, -1e30)).ravel()
    np.testing.assert_allclose(y, [1, 2, 1, 2], atol=1e-3)


def test_fused_attention_full_mask_broadcasts_and_fully_masked_rows(port):
    rng = np.random.default_rng(1)
    B, S, H = 2, 96, 128
    q, k, v = [rng.standard_normal((B, S, H), dtype=np.float32) for _ in range(3)]
    m = (rng.random((B, 2, S, S)) < 0.3).astype(np.uint8)  # per-head, per-query mask
    m[1, 0, 5, :] = 1  # fully masked row -> uniform weights
    y = host(ops.FusedAttention(T(q), T(k), T(v), T(m), 64, -3.0e38))
    np.testing.assert_allclose(y, port.fused_attention(q, k, v, m, 64, -3.0e38), atol=2e-5)
    with pytest.raises(RuntimeError, match="broadcast"):
        ops.FusedAttention(T(q), T(k), T(v), T(np.zeros((3, 1, 1, S), np.uint8)), 64, -3.0e38)


def test_fused_attention_head_dim_32_generic(port):
    q, k, v, m = _attn_case(2, 40, 96, 32, [40, 20], 3)
    y = host(ops.FusedAttention(T(q), T(k), T(v), T(m), 32, -3.0e38))
    np.testing.assert_allclose(y, port.fused_attention(q, k, v, m, 32, -3.0e38), atol=2e-5)


# ------------------------------------------------------------ pointwise

def test_gelu_gelu_tanh_softmax_golden(gold):
    g, i = gold
    np.testing.assert_allclose(host(ops.GeluTanh(T(i["gt_x"]))), g["gt_y"], atol=1e-6)
    np.testing.assert_allclose(host(ops.Gelu(T(i["gt_x"]))), g["ge_y"], atol=1e-6)
    np.testing.assert_allclose(host(ops.Softmax(T(i["sm_x"]))), g["sm_y"], atol=1e-7)
    x = T(np.array([[1000, 1001, 999, 1002]], np.float32))
    y = host(ops.Softmax(x))
    assert np.isfinite(y).all() and abs(y.sum() - 1) < 1e-5


# ------------------------------------------------------------ decode ops

@pytest.mark.parametrize("K,Nn,act", [(768, 2304, None), (768, 3072, "gelu_tanh"),
                                      (3072, 768, None), (768, 768, None), (100, 50, "relu"),
                                      (768, 50, None)])
def test_gemv_kn(port, K, Nn, act):
    rng = np.random.default_rng(K + Nn)
    x = rng.standard_normal(K, dtype=np.float32)
    w = (rng.standard_normal((K, Nn), dtype=np.float32) * 0.02).astype(np.float32)
    b = rng.standard_normal(Nn, dtype=np.float32) * 0.1
    r = rng.standard_normal(Nn, dtype=np.float32)
    for _ in range(2):  # second call checks the split-K counters were reset
        y = host(ops.Gemv(T(x), T(w), T(b), T(r), act))
    ref = port.gemm(x[None], w, b) + r
    if act == "gelu_tanh":
        ref = port.gelu_tanh(ref)
    elif act == "relu":
        ref = np.maximum(ref, 0)
    np.testing.assert_allclose(y, ref.ravel(), atol=1e-5, rtol=1e-5)


def test_gemv_is_deterministic():
    rng = np.random.default_rng(0)
    x = T(rng.standard_normal(3072, dtype=np.float32))
    w = T(rng.standard_normal((3072, 768), dtype=np.float32))
    outs = [host(ops.Gemv(x, w)) for _ in range(5)]
    for o in outs[1:]:
        np.testing.assert_array_equal(o, outs[0])


def test_argmax_first_max_wins():
    x = torch.zeros(50257, device=DEV)
    x[[7, 30000, 50256]] = 3.0
    assert int(ops.Argmax(x)) == 7
    x = torch.randn(50257, device=DEV)
    assert int(ops.Argmax(x)) == int(torch.argmax(x))
    assert int(ops.Argmax(torch.tensor([2.0], device=DEV))) == 0


@pytest.mark.parametrize("n,k", [(16, 256), (2304, 768), (768, 3072), (50257, 768), (37, 130),
                                 (5, 2)])
def test_int4_rowscale(port, n, k):
    rng = np.random.default_rng(n + k)
    m = synth.int4_matrix(n, k, rng)
    y = host(ops.Int4GemvRowScale(T(m.w), T(m.scales), T(m.x)))
    ref = port.int4_gemv_rowscale(m.w, m.scales, m.x)
    tol = 1e-6 * np.abs(m.scales).max() * np.abs(m.x).sum() * 8 + 1e-6
    np.testing.assert_allclose(y, ref, atol=tol, rtol=1e-5)


def test_int4_reference_fixture(port):
    # int4_gemv_amx.cc:481-540 fixture
    N_, K = 16, 256
    w = np.array([(i * 31) & 0xFF for i in range(N_ * K // 2)], np.uint8).reshape(N_, K // 2)
    x = np.sin(0.07 * np.arange(K)).astype(np.float32)
    s = np.array([0.05 + 0.01 * (i % 7) for i in range(N_)], np.float32)
    y = host(ops.Int4GemvRowScale(T(w), T(s), T(x)))
    np.testing.assert_allclose(y, port.int4_gemv_rowscale(w, s, x), atol=1e-4)


def test_int4_batched_gpt2_set(port):
    mats = synth.gpt2_int4_set(seed=3, layers=2)
    dev = [(T(m.w), T(m.scales), T(m.x), torch.empty(m.n, device=DEV)) for m in mats]
    ops.Int4GemvBatched(dev)
    for m, d in zip(mats, dev):
        ref = port.int4_gemv_rowscale(m.w, m.scales, m.x)
        np.testing.assert_allclose(host(d[3]), ref, atol=1e-4, rtol=1e-5)


def test_int4_batched_many_small_and_mixed(port):
    """70 matrices of mixed shapes in one call: more than one launch pair,
    many matrix switches inside each CTA, tails of K below one 256-weight
    slab, a K that is not a multiple of 32 (the per-row kernel), and x of very
    different magnitudes per matrix (each has its own activation scale)."""
    rng = np.random.default_rng(17)
    shapes = [(int(rng.integers(1, 300)), int(rng.choice([32, 64, 96, 768, 1024, 4096])))
              for _ in range(68)] + [(129, 130), (3, 4096)]
    mats = []
    for i, (n, k) in enumerate(shapes):
        m = synth.int4_matrix(n, k, rng)
        m = synth.Int4Matrix(m.w, m.scales, (m.x * 10.0 ** ((i % 7) - 3)).astype(np.float32))
        mats.append(m)
    dev = [(T(m.w), T(m.scales), T(m.x), torch.empty(m.n, device=DEV)) for m in mats]
    ops.Int4GemvBatched(dev)
    for m, d in zip(mats, dev):
        ref = port.int4_gemv_rowscale(m.w, m.scales, m.x)
        tol = 1e-6 * np.abs(m.scales).max() * np.abs(m.x).sum() * 8 + 1e-30
        np.testing.assert_allclose(host(d[3]), ref, atol=tol, rtol=1e-5)


@pytest.mark.parametrize("n,k", [(128, 4096), (200, 4096), (300, 2048), (5, 1024)])
def test_int4_split_blocks_repeat(port, n, k):
    """Few blocks with many slabs: the grid is one CTA per slab or so, so
    every 128-row block is summed by several CTAs through the partial-sum
    scratch. Three calls in a row must agree bit for bit (the scratch returns
    to zero after each launch) and match the port."""
    rng = np.random.default_rng(n * 7 + k)
    m = synth.int4_matrix(n, k, rng)
    ref = port.int4_gemv_rowscale(m.w, m.scales, m.x)
    outs = []
    for _ in range(3):
        y = host(ops.Int4GemvRowScale(T(m.w), T(m.scales), T(m.x)))
        np.testing.assert_allclose(y, ref, atol=1e-4, rtol=1e-5)
        outs.append(y)
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])


@pytest.mark.parametrize("B,S", [(2, 128), (1, 512), (3, 40)])
def test_qkv_attention_prepared(port, B, S):
    """inferc_dev_qkv_attention (config 2 path) == FusedQKV + FusedAttention."""
    import ctypes  # noqa: F401
    from inferc_b200 import lib
    L = lib.load()
    x, ws, lens = synth.attention_sweep_inputs(B, S, seed=B + S)
    H = 768
    wcat = np.ascontiguousarray(np.concatenate([ws[0], ws[2], ws[4]], axis=1))
    bcat = np.concatenate([ws[1], ws[3], ws[5]]).astype(np.float32)
    wd = T(wcat)
    wb, wsm = torch.empty_like(wd), torch.empty_like(wd)
    lib.check(L.inferc_dev_tf32_split(wd.data_ptr(), wb.data_ptr(), wsm.data_ptr(), wd.numel(),
                                      None))
    km = (np.arange(S)[None, :] >= lens[:, None]).astype(np.uint8)
    scratch = torch.empty(B * S * 3 * H, device=DEV)
    out = torch.empty(B, S, H, device=DEV)
    xd, bd, md = T(x), T(bcat), T(km)
    lib.check(L.inferc_dev_qkv_attention(xd.data_ptr(), wb.data_ptr(), wsm.data_ptr(),
                                         bd.data_ptr(), md.data_ptr(), B, S, H, 64, -3.0e38,
                                         scratch.data_ptr(), out.data_ptr(), None))
    q, k, v = port.fused_qkv(x.reshape(B * S, H), ws[0], ws[1], ws[2], ws[3], ws[4], ws[5])
    ref = port.fused_attention(q.reshape(B, S, H), k.reshape(B, S, H), v.reshape(B, S, H),
                               km.reshape(B, 1, 1, S), 64, -3.0e38)
    np.testing.assert_allclose(host(out), ref, atol=5e-5)


@pytest.mark.parametrize("B,S", [(1, 128), (8, 128), (3, 70), (1, 1), (2, 17), (4, 100),
                                 (2, 512), (1, 300), (3, 257),
                                 (64, 128), (31, 97)])
def test_fused_attention_planes(port, B, S):
    """Split-fp16 tensor-core attention on q, k, v planes cut from one
    [B*S, 3H] pair (the encoder plan's layout), against the reference; S > 128
    runs the flash form (online softmax over 128-key blocks)."""
    from inferc_b200 import lib
    L = lib.load()
    H = 768
    lens = np.random.default_rng(B * S + 1).integers(1, S + 1, size=B)
    q, k, v, m = _attn_case(B, S, H, 64, lens, B + S + 7)
    qkv = np.concatenate([q, k, v], axis=2).reshape(B * S, 3 * H)
    x = T(qkv)
    hi, lo = (torch.empty((B * S, 3 * H), dtype=torch.int16, device=DEV) for _ in range(2))
    lib.check(L.inferc_dev_f16_split_rows(x.data_ptr(), B * S, 3 * H, 3 * H, hi.data_ptr(),
                                          lo.data_ptr(), 3 * H, None))
    out = torch.empty((B, S, H), device=DEV)
    km = T(m.reshape(B, S))
    e = 2  # bytes per int16
    lib.check(L.inferc_dev_fused_attention_planes(
        hi.data_ptr(), lo.data_ptr(), hi.data_ptr() + H * e, lo.data_ptr() + H * e,
        hi.data_ptr() + 2 * H * e, lo.data_ptr() + 2 * H * e, 3 * H, km.data_ptr(), B, S, 12,
        -3.4028234663852886e38, out.data_ptr(), None))
    lib.check(L.inferc_dev_stream_synchronize(None))
    ref = port.fused_attention(q, k, v, m, 64, -3.4028234663852886e38)
    np.testing.assert_allclose(host(out), ref, atol=2e-5)


@pytest.mark.parametrize("S,lens", [(300, [0, 5, 300]), (512, [1, 129, 256, 257]),
                                    (700, [700, 0, 64])])
def test_fused_attention_planes_masked_blocks(port, S, lens):
    """The flash form skips key blocks whose keys are all masked (exact zeros
    in the sums); a sequence with no visible key keeps every block and gets
    the reference's uniform weights."""
    from inferc_b200 import lib
    L = lib.load()
    H, B = 768, len(lens)
    q, k, v, m = _attn_case(B, S, H, 64, np.array(lens), S + 11)
    qkv = np.concatenate([q, k, v], axis=2).reshape(B * S, 3 * H)
    x = T(qkv)
    hi, lo = (torch.empty((B * S, 3 * H), dtype=torch.int16, device=DEV) for _ in range(2))
    lib.check(L.inferc_dev_f16_split_rows(x.data_ptr(), B * S, 3 * H, 3 * H, hi.data_ptr(),
                                          lo.data_ptr(), 3 * H, None))
    out = torch.empty((B, S, H), device=DEV)
    km = T(m.reshape(B, S))
    e = 2
    lib.check(L.inferc_dev_fused_attention_planes(
        hi.data_ptr(), lo.data_ptr(), hi.data_ptr() + H * e, lo.data_ptr() + H * e,
        hi.data_ptr() + 2 * H * e, lo.data_ptr() + 2 * H * e, 3 * H, km.data_ptr(), B, S, 12,
        -3.4028234663852886e38, out.data_ptr(), None))
    lib.check(L.inferc_dev_stream_synchronize(None))
    ref = port.fused_attention(q, k, v, m, 64, -3.4028234663852886e38)
    np.testing.assert_allclose(host(out), ref, atol=2e-5)


@pytest.mark.parametrize("B,S", [(2, 128), (1, 512), (3, 40)])
def test_qkv_attention_f16(port, B, S):
    """inferc_dev_qkv_attention_f16 (split-fp16 weights, planes end to end) ==
    FusedQKV + FusedAttention of the reference."""
    from inferc_b200 import lib
    L = lib.load()
    x, ws, lens = synth.attention_sweep_inputs(B, S, seed=B + S + 3)
    H = 768
    wcat = T(np.ascontiguousarray(np.concatenate([ws[0], ws[2], ws[4]], axis=1)))
    bcat = T(np.concatenate([ws[1], ws[3], ws[5]]).astype(np.float32))
    kp = L.inferc_dev_f16_kp(H)
    wh, wl = (torch.empty((3 * H, kp), dtype=torch.int16, device=DEV) for _ in range(2))
    sc = torch.empty(2, device=DEV)
    lib.check(L.inferc_dev_f16_split(wcat.data_ptr(), H, 3 * H, 3 * H, wh.data_ptr(),
                                     wl.data_ptr(), sc.data_ptr(), None))
    km = (np.arange(S)[None, :] >= lens[:, None]).astype(np.uint8)
    scratch = torch.empty(8 * B * S * H, dtype=torch.int16, device=DEV)
    out = torch.empty(B, S, H, device=DEV)
    xd, md = T(x), T(km)
    lib.check(L.inferc_dev_qkv_attention_f16(xd.data_ptr(), wh.data_ptr(), wl.data_ptr(),
                                             sc.data_ptr(), bcat.data_ptr(), md.data_ptr(), B, S,
                                             H, 64, -3.0e38, scratch.data_ptr(), out.data_ptr(),
                                             None))
    lib.check(L.inferc_dev_stream_synchronize(None))
    q, k, v = port.fused_qkv(x.reshape(B * S, H), ws[0], ws[1], ws[2], ws[3], ws[4], ws[5])
    ref = port.fused_attention(q.reshape(B, S, H), k.reshape(B, S, H), v.reshape(B, S, H),
                               km.reshape(B, 1, 1, S), 64, -3.0e38)
    np.testing.assert_allclose(host(out), ref, atol=5e-5)


def test_empty_inputs():
    """Zero rows, batch or sequence length. The reference kernels' loops run
    zero times and return empty tensors; every entry here returns status 0
    without a launch, and the outputs keep their shapes."""
    def z(*s):
        return torch.zeros(*s, device=DEV)

    assert ops.FusedMatMulAddGELU(z(0, 768), z(768, 3072), z(3072)).shape == (0, 3072)
    outs = ops.FusedQKVProjection(z(0, 4, 768), z(768, 768), z(768), z(768, 768), z(768),
                                  z(768, 768), z(768))
    assert [tuple(o.shape) for o in outs] == [(0, 4, 768)] * 3
    assert ops.LayerNorm(z(0, 768), z(768) + 1, z(768)).shape == (0, 768)
    assert ops.Gemm(z(0, 4), z(4, 5)).shape == (0, 5)
    assert ops.FusedAttention(z(0, 128, 768), z(0, 128, 768), z(0, 128, 768)).shape == (0, 128, 768)
    assert ops.FusedAttention(z(2, 0, 768), z(2, 0, 768), z(2, 0, 768)).shape == (2, 0, 768)
    w = torch.zeros(0, 384, dtype=torch.uint8, device=DEV)
    assert ops.Int4GemvRowScale(w, z(0), z(768)).shape == (0,)
    ops.Int4GemvBatched([])
    torch.cuda.synchronize()
