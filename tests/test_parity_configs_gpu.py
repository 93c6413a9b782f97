"""Parity at the shapes bench.py times, checked against the reference's own
CPU kernels (oracle/_ref, built from the reference sources; the C
restatement stands in where that build is absent):

  - C4: all 256 sequences of the batch-256 variable-length workload against
    the reference logits committed in tests/golden/encoder_c4_bench.npz;
  - C2: every (seq, batch) point of the QKV + attention sweep at the bench's
    seeds, four sampled sequences per point (sequences are independent);
  - C3: the full 49-matrix int4 set in one batched call;
  - C1: the per-kernel CUDA-graph decode step (the fallback for shapes the
    persistent kernel does not take) on the full GPT-2-small config, and the
    op-level KV-append / decode-attention entries.
"""
import os

import numpy as np
import pytest
import torch

from inferc_b200 import lib, ops, plans, synth
from oracle import oracle

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LOGIT_TOL = 1e-4  # north-star tolerance on fp32 logits
FILL = -3.4028234663852886e38


def _ref():
    return oracle.ref() or oracle.port()


def test_c4_all_256_sequences_of_the_bench_workload():
    gold = np.load(os.path.join(GOLD, "encoder_c4_bench.npz"))
    cfg = synth.EncoderConfig()
    ids, mask = synth.encoder_inputs(256, 128, seed=int(gold["seed"]), variable_lengths=True)
    p = plans.EncoderPlan(cfg, synth.encoder_weights(cfg, seed=0), max_batch=256, max_seq=128)
    got = p.run_host(ids, mask)
    err = np.abs(got - gold["logits"]).max(axis=1)
    lens = mask.sum(1)
    # every length bucket of the workload is covered by the comparison
    assert len(np.unique(np.digitize(lens, [32, 64, 96]))) == 4
    assert err.max() <= LOGIT_TOL, (err.max(), int(err.argmax()), int(lens[err.argmax()]))
    assert (got.argmax(1) == gold["logits"].argmax(1)).all()
    ffb = lib.load().inferc_dev_encoder_range_fallbacks(p._h)
    assert ffb == 0


@pytest.mark.parametrize("S", [128, 512])
@pytest.mark.parametrize("B", [1, 8, 64])
def test_c2_sweep_point(S, B):
    """inferc_dev_qkv_attention_f16 at the bench's inputs (attention_sweep_inputs
    default seed) vs FusedQKVProjection + FusedAttention of the reference on
    four sampled sequences."""
    L = lib.load()
    H = 768
    x, ws, lens = synth.attention_sweep_inputs(B, S)
    wcat = torch.from_numpy(np.ascontiguousarray(np.concatenate([ws[0], ws[2], ws[4]], 1))).cuda()
    bcat = torch.from_numpy(np.concatenate([ws[1], ws[3], ws[5]]).astype(np.float32)).cuda()
    kp = L.inferc_dev_f16_kp(H)
    wh, wl = (torch.empty((3 * H, kp), dtype=torch.int16, device="cuda") for _ in range(2))
    sc = torch.empty(2, device="cuda")
    lib.check(L.inferc_dev_f16_split(wcat.data_ptr(), H, 3 * H, 3 * H, wh.data_ptr(),
                                     wl.data_ptr(), sc.data_ptr(), None))
    km = (np.arange(S)[None, :] >= lens[:, None]).astype(np.uint8)
    xd, md = torch.from_numpy(x).cuda(), torch.from_numpy(km).cuda()
    scratch = torch.empty(8 * B * S * H, dtype=torch.int16, device="cuda")
    out = torch.empty(B, S, H, device="cuda")
    lib.check(L.inferc_dev_qkv_attention_f16(xd.data_ptr(), wh.data_ptr(), wl.data_ptr(),
                                             sc.data_ptr(), bcat.data_ptr(), md.data_ptr(), B, S,
                                             H, 64, FILL, scratch.data_ptr(), out.data_ptr(),
                                             None))
    lib.check(L.inferc_dev_stream_synchronize(None))
    got = out.cpu().numpy()
    ref = _ref()
    picks = sorted({0, B - 1, B // 2, B // 3})
    for b in picks:
        q, k, v = ref.fused_qkv(x[b].reshape(S, H), *ws)
        want = ref.fused_attention(q.reshape(1, S, H), k.reshape(1, S, H), v.reshape(1, S, H),
                                   km[b].reshape(1, 1, 1, S), 64, FILL)[0]
        np.testing.assert_allclose(got[b], want, atol=5e-5, err_msg=f"sequence {b}")


def test_c3_full_int4_set_one_call():
    port = oracle.port()
    mats = synth.gpt2_int4_set(seed=3)
    assert len(mats) == 49
    dev = [(torch.from_numpy(m.w).cuda(), torch.from_numpy(m.scales).cuda(),
            torch.from_numpy(m.x).cuda(), torch.empty(m.n, device="cuda")) for m in mats]
    ops.Int4GemvBatched(dev)
    torch.cuda.synchronize()
    for i, (m, d) in enumerate(zip(mats, dev)):
        want = port.int4_gemv_rowscale(m.w, m.scales, m.x)
        tol = 1e-6 * np.abs(m.scales).max() * np.abs(m.x).sum() * 8 + 1e-6
        np.testing.assert_allclose(d[3].cpu().numpy(), want, atol=tol, rtol=1e-5,
                                   err_msg=f"matrix {i}")


def test_c1_decode_graph_step_full_config(monkeypatch):
    """INFERC_DECODE_GRAPH=1: every single-token step replays the 62-launch
    CUDA graph instead of the persistent kernel; tokens still bit-identical
    to the reference on the full 32 + 128 token workload."""
    gold = np.load(os.path.join(GOLD, "decode.npz"))
    monkeypatch.setenv("INFERC_DECODE_GRAPH", "1")
    cfg = synth.Gpt2Config()
    p = plans.DecoderPlan(cfg, synth.gpt2_weights(cfg, seed=0), max_len=1024)
    toks, ms = p.decode(gold["c1_prompt"], 128)
    np.testing.assert_array_equal(toks, gold["c1_tokens"])
    assert ms > 0


def _np_decode_attention(q, kc, vc, L, heads, hd):
    out = np.empty(heads * hd, np.float64)
    for h in range(heads):
        qh = q[h * hd:(h + 1) * hd].astype(np.float64)
        s = kc[h, :L].astype(np.float64) @ qh / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * hd:(h + 1) * hd] = p @ vc[h, :L].astype(np.float64)
    return out.astype(np.float32)


@pytest.mark.parametrize("L,n", [(1, 1), (33, 32), (160, 1), (1000, 7)])
def test_kv_append_and_decode_attention_entries(L, n):
    """inferc_dev_kv_append writes n new K/V rows at positions [L-n, L) of a
    [heads, max_len, hd] cache (the with-past graph's Concat,
    src/kernels/movement.cc:142-189); inferc_dev_decode_attention then
    attends one query over the first L positions (MatMul, Div, Softmax,
    MatMul of the decode step)."""
    Lb = lib.load()
    heads, hd, max_len = 12, 64, 1024
    rng = np.random.default_rng(L * 3 + n)
    kc = rng.standard_normal((heads, max_len, hd), dtype=np.float32)
    vc = rng.standard_normal((heads, max_len, hd), dtype=np.float32)
    knew = rng.standard_normal((n, heads * hd), dtype=np.float32)
    vnew = rng.standard_normal((n, heads * hd), dtype=np.float32)
    q = rng.standard_normal(heads * hd, dtype=np.float32)
    kd, vd = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    knd, vnd, qd = (torch.from_numpy(a).cuda() for a in (knew, vnew, q))
    out = torch.empty(heads * hd, device="cuda")
    pos = L - n
    lib.check(Lb.inferc_dev_kv_append(knd.data_ptr(), vnd.data_ptr(), heads * hd, kd.data_ptr(),
                                      vd.data_ptr(), heads, hd, max_len, pos, n, None))
    lib.check(Lb.inferc_dev_decode_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(),
                                             out.data_ptr(), heads, hd, max_len, L, None))
    torch.cuda.synchronize()
    for r in range(n):
        kc[:, pos + r] = knew[r].reshape(heads, hd)
        vc[:, pos + r] = vnew[r].reshape(heads, hd)
    np.testing.assert_array_equal(kd.cpu().numpy(), kc)
    np.testing.assert_array_equal(vd.cpu().numpy(), vc)
    np.testing.assert_allclose(out.cpu().numpy(), _np_decode_attention(q, kc, vc, L, heads, hd),
                               atol=2e-5, rtol=1e-5)
    # bad arguments are rejected, not run
    assert Lb.inferc_dev_kv_append(knd.data_ptr(), vnd.data_ptr(), heads * hd, kd.data_ptr(),
                                   vd.data_ptr(), heads, hd, max_len, max_len, 1, None) == 1
    assert Lb.inferc_dev_decode_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(),
                                          out.data_ptr(), heads, hd, max_len, max_len + 1,
                                          None) == 1
