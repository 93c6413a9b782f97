"""Tensor-core (tcgen05, 3xTF32) GEMM: fp32-level accuracy against a float64
reference across tile-aligned and ragged shapes, with each epilogue."""
import numpy as np
import pytest
import torch

from inferc_b200 import ops

pytestmark = pytest.mark.gpu

# Max error relative to max |C| at K <= 3072. Sequential fp32 reaches ~2e-6
# there; the tensor core's fp32 accumulation adds a K-proportional term
# (measured 2e-5 at K=3072), still ~30x below plain TF32 (~1e-3 rel).
TC_REL_TOL = 3e-5


def _rel_err(got, ref):
    return float(np.abs(got - ref).max() / (np.abs(ref).max() + 1e-30))


@pytest.mark.parametrize("M,K,N", [(256, 64, 256), (256, 768, 3072), (512, 3072, 768),
                                   (300, 100, 200), (4096, 768, 2304), (257, 36, 33)])
def test_tc_matmul_fp32_accuracy(M, K, N):
    rng = np.random.default_rng(M + K + N)
    a = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal((K, N), dtype=np.float32)
    y = ops.MatMul(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    torch.cuda.synchronize()
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert _rel_err(y.cpu().numpy(), ref) < TC_REL_TOL


def test_tc_fused_gelu_and_bias_residual():
    rng = np.random.default_rng(0)
    M, K, N = 1024, 768, 3072
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = (rng.standard_normal((K, N), dtype=np.float32) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N, dtype=np.float32) * 0.1).astype(np.float32)
    y = ops.FusedMatMulAddGELU(*(torch.from_numpy(t).cuda() for t in (x, w, b)))
    torch.cuda.synchronize()
    v = x.astype(np.float64) @ w.astype(np.float64) + b
    from math import erf, sqrt
    ref = v * 0.5 * (1 + np.vectorize(lambda t: erf(t / sqrt(2)))(v))
    assert np.abs(y.cpu().numpy() - ref).max() < 3e-5
    c = rng.standard_normal((M, N), dtype=np.float32)
    g = ops.Gemm(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(),
                 torch.from_numpy(c).cuda(), 0.5, 2.0)
    torch.cuda.synchronize()
    ref = 0.5 * (x.astype(np.float64) @ w.astype(np.float64)) + 2.0 * c
    assert _rel_err(g.cpu().numpy(), ref) < TC_REL_TOL


def test_prepared_weight_entry_points():
    """inferc_dev_tf32_split + inferc_dev_gemm_tf32x3 (prepared weights), both
    the tensor-core shape and the small-M CUDA-core shape, with an in-place
    residual."""
    from inferc_b200 import lib
    L = lib.load()
    rng = np.random.default_rng(2)
    for M in (512, 40):
        K, N = 768, 768
        a = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
        w = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32) * 0.05).cuda()
        b = torch.from_numpy(rng.standard_normal(N, dtype=np.float32)).cuda()
        r = torch.from_numpy(rng.standard_normal((M, N), dtype=np.float32)).cuda()
        big, small = torch.empty_like(w), torch.empty_like(w)
        lib.check(L.inferc_dev_tf32_split(w.data_ptr(), big.data_ptr(), small.data_ptr(),
                                          w.numel(), None))
        y = r.clone()
        lib.check(L.inferc_dev_gemm_tf32x3(a.data_ptr(), K, big.data_ptr(), small.data_ptr(), N,
                                           b.data_ptr(), y.data_ptr(), N, y.data_ptr(), N, M, N,
                                           K, 1, None))
        torch.cuda.synchronize()
        v = a.double() @ w.double() + b.double() + r.double()
        ref = (v * 0.5 * (1 + torch.erf(v / 2 ** 0.5))).cpu().numpy()
        assert np.abs(y.cpu().numpy() - ref).max() < 5e-5
