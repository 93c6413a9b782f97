"""The allocation-free GEMV entry point, inferc_dev_gemv_noalloc, is for
callers that may not allocate device memory themselves or through the
library (a host framework that owns the device heap, an allocator-less
runtime, a real-time loop). It must give the same result as
inferc_dev_gemv on the same inputs, call after call, while taking its
scratch from the array built into the library.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test."""
import numpy as np
import pytest
import torch

from inferc_b200 import lib

pytestmark = pytest.mark.gpu


def _call(name, x, w, b, r, y, act):
    L = lib.load()
    K, N = w.shape
    rc = getattr(L, name)(x.data_ptr(), w.data_ptr(), None if b is None else b.data_ptr(),
                          None if r is None else r.data_ptr(), y.data_ptr(), K, N, act,
                          torch.cuda.current_stream().cuda_stream)
    lib.check(rc)


@pytest.mark.parametrize("K,N,act", [(768, 2304, 0), (3072, 768, 0), (768, 3072, 2),
                                     (768, 50, 3), (8192, 1024, 0), (8192, 2048, 3), (8192, 4096, 1)])
def test_noalloc_matches_gemv_twice(K, N, act):
    rng = np.random.default_rng(K * 7 + N)
    x = torch.from_numpy(rng.standard_normal(K, dtype=np.float32)).cuda()
    w = torch.from_numpy((rng.standard_normal((K, N), dtype=np.float32) * 0.02)).cuda()
    b = torch.from_numpy(rng.standard_normal(N, dtype=np.float32)).cuda()
    r = torch.from_numpy(rng.standard_normal(N, dtype=np.float32)).cuda()
    want = torch.empty(N, device="cuda")
    _call("inferc_dev_gemv", x, w, b, r, want, act)
    for _ in range(2):  # the shared scratch must be reusable call after call
        got = torch.full((N,), float("nan"), device="cuda")
        _call("inferc_dev_gemv_noalloc", x, w, b, r, got, act)
        torch.cuda.synchronize()
        # Both entry points pick the split-K count by one rule, so they sum in
        # the same order and agree bit for bit, unless the built-in 1 MiB
        # scratch caps the split count (splits x N partial sums must fit):
        # then the order differs and they agree within fp32 rounding.
        splits = max(-(-K // 64), 1)
        if splits * N <= (1 << 18):
            np.testing.assert_array_equal(got.cpu().numpy(), want.cpu().numpy())
        else:
            np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), atol=1e-5,
                                       rtol=1e-5)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    x = torch.zeros(8, device="cuda")
    w = torch.zeros(8, 4, device="cuda")
    y = torch.zeros(4, device="cuda")
    L = lib.load()
    rc = L.inferc_dev_gemv_noalloc(x.data_ptr(), w.data_ptr(), None, None, y.data_ptr(), 8,
                                   (1 << 18) + 4, 0, None)
    assert rc == 1 and b"scratch" in L.inferc_dev_last_error_string()
