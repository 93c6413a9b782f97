"""Split-fp16 tensor-core GEMM (tcgen05 kind::f16, three MMAs per product):
fp32-level accuracy against a float64 reference on tile-aligned and ragged
shapes, each epilogue, weights of very different scales, and the range flag
raised by an activation that fp16 cannot carry."""
import numpy as np
import pytest
import torch

from inferc_b200 import lib

pytestmark = pytest.mark.gpu

# Same bar as the 3xTF32 kernel: max error relative to max |C| (the tensor
# core's fp32 accumulation dominates, ~2e-5 at K=3072).
TC_REL_TOL = 3e-5


def _prep(L, w):
    K, N = w.shape
    kp = L.inferc_dev_f16_kp(K)
    hi = torch.empty((N, kp), dtype=torch.int16, device="cuda")
    lo = torch.empty((N, kp), dtype=torch.int16, device="cuda")
    sc = torch.empty(2, dtype=torch.float32, device="cuda")
    lib.check(L.inferc_dev_f16_split(w.data_ptr(), K, N, N, hi.data_ptr(), lo.data_ptr(),
                                     sc.data_ptr(), None))
    return hi, lo, sc


def _gemm(L, a, prep, N, bias=None, resid=None, act=0):
    hi, lo, sc = prep
    M, K = a.shape
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    lib.check(L.inferc_dev_gemm_f16s(a.data_ptr(), K, hi.data_ptr(), lo.data_ptr(), sc.data_ptr(),
                                     bias.data_ptr() if bias is not None else None,
                                     resid.data_ptr() if resid is not None else None, N,
                                     y.data_ptr(), N, M, N, K, act, None))
    return y


def _rel_err(got, ref):
    return float(np.abs(got - ref).max() / (np.abs(ref).max() + 1e-30))


@pytest.mark.parametrize("M,K,N", [(256, 64, 256), (256, 768, 3072), (512, 3072, 768),
                                   (300, 100, 200), (4096, 768, 2304), (257, 36, 33),
                                   (1, 768, 768), (32768, 768, 768)])
def test_f16s_fp32_accuracy(M, K, N):
    L = lib.load()
    rng = np.random.default_rng(M + K + N)
    a = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((K, N), dtype=np.float32) * 0.02).astype(np.float32)
    ta, tw = torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda()
    y = _gemm(L, ta, _prep(L, tw), N)
    lib.check(L.inferc_dev_stream_synchronize(None))
    ref = (ta.double() @ tw.double()).cpu().numpy()
    assert _rel_err(y.cpu().numpy(), ref) < TC_REL_TOL


@pytest.mark.parametrize("wscale,ascale", [(1e-4, 1.0), (30.0, 1e-3), (0.02, 100.0)])
def test_f16s_operand_scales(wscale, ascale):
    """Small and large weights (the power-of-two prescale) and activations far
    from 1 (small ones lean on fp16 subnormals for lo)."""
    L = lib.load()
    rng = np.random.default_rng(7)
    M, K, N = 512, 768, 512
    a = (rng.standard_normal((M, K)) * ascale).astype(np.float32)
    w = (rng.standard_normal((K, N)) * wscale).astype(np.float32)
    ta, tw = torch.from_numpy(a).cuda(), torch.from_numpy(w).cuda()
    y = _gemm(L, ta, _prep(L, tw), N)
    lib.check(L.inferc_dev_stream_synchronize(None))
    ref = (ta.double() @ tw.double()).cpu().numpy()
    assert _rel_err(y.cpu().numpy(), ref) < TC_REL_TOL


def test_f16s_epilogues():
    L = lib.load()
    rng = np.random.default_rng(3)
    M, K, N = 1024, 768, 3072
    a = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
    w = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32) * 0.02).cuda()
    b = torch.from_numpy(rng.standard_normal(N, dtype=np.float32) * 0.1).cuda()
    r = torch.from_numpy(rng.standard_normal((M, N), dtype=np.float32)).cuda()
    prep = _prep(L, w)
    v = a.double() @ w.double() + b.double()
    y = _gemm(L, a, prep, N, bias=b, act=1)
    ref = v * 0.5 * (1 + torch.erf(v / 2 ** 0.5))
    assert (y.double() - ref).abs().max().item() < 3e-5
    y = _gemm(L, a, prep, N, bias=b, resid=r)
    assert (y.double() - (v + r.double())).abs().max().item() < 3e-5
    lib.check(L.inferc_dev_stream_synchronize(None))


def test_f16s_range_flag():
    """An activation beyond fp16's range is reported at the next synchronize
    (INFERC_ERR_RANGE) and the flag is cleared; a following in-range call is
    clean again."""
    L = lib.load()
    rng = np.random.default_rng(5)
    M, K, N = 256, 128, 256
    a = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
    w = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32)).cuda()
    prep = _prep(L, w)
    bad = a.clone()
    bad[17, 5] = 1.0e6
    _gemm(L, bad, prep, N)
    assert L.inferc_dev_stream_synchronize(None) == 5
    y = _gemm(L, a, prep, N)
    lib.check(L.inferc_dev_stream_synchronize(None))
    ref = (a.double() @ w.double()).cpu().numpy()
    assert _rel_err(y.cpu().numpy(), ref) < TC_REL_TOL


def test_f16s_planes_chain():
    """The encoder plan's FFN chain through the plane entry points: x split by
    inferc_dev_f16_split_rows, FFN1 (bias + GELU) storing its fp16 split, FFN2
    reading that split with bias + residual; against float64."""
    L = lib.load()
    rng = np.random.default_rng(11)
    M, H, F = 1000, 768, 3072
    x = torch.from_numpy(rng.standard_normal((M, H), dtype=np.float32)).cuda()
    w1 = torch.from_numpy(rng.standard_normal((H, F), dtype=np.float32) * 0.02).cuda()
    b1 = torch.from_numpy(rng.standard_normal(F, dtype=np.float32) * 0.02).cuda()
    w2 = torch.from_numpy(rng.standard_normal((F, H), dtype=np.float32) * 0.02).cuda()
    b2 = torch.from_numpy(rng.standard_normal(H, dtype=np.float32) * 0.02).cuda()
    p1, p2 = _prep(L, w1), _prep(L, w2)
    xh, xl = (torch.empty((M, H), dtype=torch.int16, device="cuda") for _ in range(2))
    hh, hl = (torch.empty((M, F), dtype=torch.int16, device="cuda") for _ in range(2))
    lib.check(L.inferc_dev_f16_split_rows(x.data_ptr(), M, H, H, xh.data_ptr(), xl.data_ptr(), H,
                                          None))
    lib.check(L.inferc_dev_gemm_f16s_planes(xh.data_ptr(), xl.data_ptr(), H, p1[0].data_ptr(),
                                            p1[1].data_ptr(), p1[2].data_ptr(), b1.data_ptr(),
                                            None, 0, None, hh.data_ptr(), hl.data_ptr(), F, M, F,
                                            H, 1, None))
    y = torch.empty((M, H), device="cuda")
    lib.check(L.inferc_dev_gemm_f16s_planes(hh.data_ptr(), hl.data_ptr(), F, p2[0].data_ptr(),
                                            p2[1].data_ptr(), p2[2].data_ptr(), b2.data_ptr(),
                                            x.data_ptr(), H, y.data_ptr(), None, None, H, M, H, F,
                                            0, None))
    lib.check(L.inferc_dev_stream_synchronize(None))
    v = x.double() @ w1.double() + b1.double()
    h = v * 0.5 * (1 + torch.erf(v / 2 ** 0.5))
    # the hidden activations reconstructed from their planes
    hf = hh.view(torch.float16).double() + hl.view(torch.float16).double()
    assert (hf - h).abs().max().item() < 3e-5
    ref = h @ w2.double() + b2.double() + x.double()
    assert (y.double() - ref).abs().max().item() < 5e-5


@pytest.mark.parametrize("M,K,N", [(512, 768, 256), (1000, 768, 2304), (4096, 3072, 768),
                                   (777, 96, 300), (32768, 768, 3072), (4096, 768, 768),
                                   (8192, 768, 768), (4000, 3072, 768), (32768, 3072, 768),
                                   (128, 768, 768), (128, 3072, 768), (100, 768, 3072),
                                   (1, 768, 2)])
def test_f16s_planes_shapes(M, K, N):
    """A as fp16 planes (the plan's form) with the bias + residual epilogue
    (fp32 out), ragged M / N / K included: whole 256-column tiles take the
    shared-memory-staged epilogue, a partial last tile the per-row one."""
    L = lib.load()
    rng = np.random.default_rng(M + N)
    a = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
    w = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32) * 0.02).cuda()
    b = torch.from_numpy(rng.standard_normal(N, dtype=np.float32)).cuda()
    r = torch.from_numpy(rng.standard_normal((M, N), dtype=np.float32)).cuda()
    hi, lo, sc = _prep(L, w)
    kp = L.inferc_dev_f16_kp(K)
    ah, al = (torch.empty((M, kp), dtype=torch.int16, device="cuda") for _ in range(2))
    lib.check(L.inferc_dev_f16_split_rows(a.data_ptr(), M, K, K, ah.data_ptr(), al.data_ptr(), kp,
                                          None))
    y = torch.empty((M, N), device="cuda")
    lib.check(L.inferc_dev_gemm_f16s_planes(ah.data_ptr(), al.data_ptr(), kp, hi.data_ptr(),
                                            lo.data_ptr(), sc.data_ptr(), b.data_ptr(),
                                            r.data_ptr(), N, y.data_ptr(), None, None, N, M, N, K,
                                            0, None))
    lib.check(L.inferc_dev_stream_synchronize(None))
    ref = a.double() @ w.double() + b.double() + r.double()
    err = (y.double() - ref).abs().max().item() / (ref.abs().max().item())
    assert err < TC_REL_TOL


@pytest.mark.parametrize("M,K,N,act", [(777, 768, 784, 1), (1000, 768, 2304, 0),
                                       (513, 3072, 272, 1), (128, 768, 2304, 0),
                                       (128, 768, 3072, 1), (77, 768, 48, 1)])
def test_f16s_split_out_shapes(M, K, N, act):
    """Split-plane output (bias, or bias + GELU) with ragged M and an N whose
    last 256-column tile is partial (staged and per-row epilogues in one
    launch); the planes' sum against float64."""
    L = lib.load()
    rng = np.random.default_rng(M * 3 + N)
    a = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
    w = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32) * 0.02).cuda()
    b = torch.from_numpy(rng.standard_normal(N, dtype=np.float32) * 0.02).cuda()
    hi, lo, sc = _prep(L, w)
    ah, al = (torch.empty((M, K), dtype=torch.int16, device="cuda") for _ in range(2))
    lib.check(L.inferc_dev_f16_split_rows(a.data_ptr(), M, K, K, ah.data_ptr(), al.data_ptr(), K,
                                          None))
    yh, yl = (torch.empty((M, N), dtype=torch.int16, device="cuda") for _ in range(2))
    lib.check(L.inferc_dev_gemm_f16s_planes(ah.data_ptr(), al.data_ptr(), K, hi.data_ptr(),
                                            lo.data_ptr(), sc.data_ptr(), b.data_ptr(), None, 0,
                                            None, yh.data_ptr(), yl.data_ptr(), N, M, N, K, act,
                                            None))
    lib.check(L.inferc_dev_stream_synchronize(None))
    v = a.double() @ w.double() + b.double()
    ref = v * 0.5 * (1 + torch.erf(v / 2 ** 0.5)) if act else v
    got = yh.view(torch.float16).double() + yl.view(torch.float16).double()
    assert (got - ref).abs().max().item() < 3e-5 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("mode", ["1", "0"])
def test_f16s_two_sm_kernel_modes(mode):
    """INFERC_GEMM_2CTA (read at process start) picks the GEMM form: "1" puts
    every eligible GEMM on the two-SM (cta_group::2, 256-row) kernel, "0"
    every GEMM on the one-SM kernel (by default split-plane outputs take the
    two-SM kernel and fp32 outputs the one-SM kernel). Run the plane and
    residual GEMM checks in a child process for each."""
    import os
    import subprocess
    import sys
    code = (
        "import sys; sys.path.insert(0, '.');"
        "from tests import test_gemm_f16s_gpu as t;"
        "t.test_f16s_planes_shapes(1000, 768, 2304); t.test_f16s_planes_shapes(512, 3072, 768);"
        "t.test_f16s_planes_chain(); print('ok')")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, INFERC_GEMM_2CTA=mode)
    out = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0 and "ok" in out.stdout, out.stderr[-2000:]
