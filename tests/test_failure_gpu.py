"""Bounded device waits give up cleanly (no trap, fault or hang): a wait on
something nothing signals runs out after a short limit, the host reads
INFERC_ERR_TIMEOUT once from inferc_dev_stream_synchronize, and the context
and the library keep working afterwards (an op call and a plan run after the
timeout still match the oracle)."""
import numpy as np
import pytest
import torch

from inferc_b200 import lib, ops
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("which", [0, 1], ids=["mbarrier", "grid-barrier"])
def test_bounded_wait_times_out_and_context_survives(which):
    L = lib.load()
    lib.check(L.inferc_dev_stream_synchronize(None))  # no stale flag
    lib.check(L.inferc_dev_selftest_wait_timeout(which, 2000, None))  # 2 ms limit
    rc = L.inferc_dev_stream_synchronize(None)
    assert rc == 4, (rc, L.inferc_dev_last_error_string())
    assert b"timed out" in L.inferc_dev_last_error_string()
    # The flag was cleared by that read.
    assert L.inferc_dev_stream_synchronize(None) == 0
    # The device still computes correctly.
    rng = np.random.default_rng(1)
    x = rng.standard_normal((64, 768), dtype=np.float32)
    g = rng.standard_normal(768, dtype=np.float32)
    b = rng.standard_normal(768, dtype=np.float32)
    y = ops.LayerNorm(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(),
                      torch.from_numpy(b).cuda(), 1e-5)
    torch.cuda.synchronize()
    np.testing.assert_allclose(y.cpu().numpy(), oracle.port().layernorm(x, g, b, 1e-5),
                               atol=1e-5, rtol=1e-5)


def test_selftest_rejects_bad_arguments():
    L = lib.load()
    assert L.inferc_dev_selftest_wait_timeout(2, 10, None) == 1
    assert L.inferc_dev_selftest_wait_timeout(0, 0, None) == 1
