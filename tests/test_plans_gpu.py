"""GPU parity of the two prepared plans against the reference:
  - encoder logits within 1e-4 (max-abs) of the reference's own kernels run
    on the same seeded model and inputs (tests/golden/encoder.npz);
  - GPT-2 greedy decode token ids bit-identical to the reference's
    (tests/golden/decode.npz), including the full GPT-2-small config
    (32-token prompt + 128 new tokens)."""
import os

import numpy as np
import pytest
import torch

from inferc_b200 import plans, synth
from inferc_b200.lib import InfercError
from oracle import oracle
from tests.golden import make_golden

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
LOGIT_TOL = 1e-4  # north-star tolerance on fp32 logits


@pytest.fixture(scope="module")
def enc_gold():
    return np.load(os.path.join(GOLD, "encoder.npz"))


@pytest.fixture(scope="module")
def dec_gold():
    return np.load(os.path.join(GOLD, "decode.npz"))


@pytest.fixture(scope="module")
def full_encoder():
    cfg = synth.EncoderConfig()
    return plans.EncoderPlan(cfg, synth.encoder_weights(cfg, seed=0), max_batch=8, max_seq=128)


def test_encoder_small_config(enc_gold):
    cfg = synth.EncoderConfig(**make_golden.SMALL_ENC)
    w = synth.encoder_weights(cfg, seed=5)
    p = plans.EncoderPlan(cfg, w, max_batch=8, max_seq=64)
    got = p.run_host(enc_gold["small_ids"], enc_gold["small_mask"])
    np.testing.assert_allclose(got, enc_gold["small_logits"], atol=LOGIT_TOL, rtol=0)


def test_encoder_c0_batch1_seq128(full_encoder, enc_gold):
    got = full_encoder.run_host(enc_gold["c0_ids"], enc_gold["c0_mask"])
    np.testing.assert_allclose(got, enc_gold["c0_logits"], atol=LOGIT_TOL, rtol=0)
    assert got.argmax(1).tolist() == enc_gold["c0_logits"].argmax(1).tolist()


def test_encoder_variable_length_batch(full_encoder, enc_gold):
    got = full_encoder.run_host(enc_gold["c4_ids"], enc_gold["c4_mask"])
    np.testing.assert_allclose(got, enc_gold["c4_logits"], atol=LOGIT_TOL, rtol=0)


def test_encoder_device_api_and_replay(full_encoder, enc_gold):
    ids = torch.from_numpy(enc_gold["c4_ids"]).cuda()
    mask = torch.from_numpy(enc_gold["c4_mask"]).cuda()
    out = torch.empty(8, 2, device="cuda")
    for _ in range(3):  # graph replays give identical results
        full_encoder.run(ids, mask, out, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), enc_gold["c4_logits"], atol=LOGIT_TOL)


def test_encoder_sub_batch_shapes(full_encoder, enc_gold):
    # A smaller (B, S) than the plan maximum gets its own graph.
    ids, mask = enc_gold["c4_ids"][:3, :64].copy(), enc_gold["c4_mask"][:3, :64].copy()
    port = oracle.port()
    cfg = synth.EncoderConfig()
    from inferc_b200 import structs
    w = synth.encoder_weights(cfg, seed=0)
    ref = port.encoder_forward(structs.encoder_struct(cfg, w), ids, mask, 2)
    np.testing.assert_allclose(full_encoder.run_host(ids, mask), ref, atol=LOGIT_TOL)


def test_encoder_tf32x3_gemm_mode(enc_gold, monkeypatch):
    """INFERC_ENCODER_GEMM=tf32x3 selects the 3xTF32 GEMMs (the split-fp16
    path's fallback) at plan creation; same logits bar."""
    monkeypatch.setenv("INFERC_ENCODER_GEMM", "tf32x3")
    cfg = synth.EncoderConfig()
    p = plans.EncoderPlan(cfg, synth.encoder_weights(cfg, seed=0), max_batch=8, max_seq=128)
    got = p.run_host(enc_gold["c4_ids"], enc_gold["c4_mask"])
    np.testing.assert_allclose(got, enc_gold["c4_logits"], atol=LOGIT_TOL, rtol=0)


def test_encoder_fp16_range_fallback():
    """Activations beyond fp16's range (embedding LayerNorm gamma = 1e5) raise
    the split-fp16 range flag; the plan reruns the batch on the 3xTF32 GEMMs
    and the logits still match the reference."""
    cfg = synth.EncoderConfig(**make_golden.SMALL_ENC)
    w = synth.encoder_weights(cfg, seed=9)
    w["emb_ln_g"] = np.full_like(w["emb_ln_g"], 1e5)
    rng = np.random.default_rng(9)
    B, S = 3, 32
    ids = rng.integers(0, cfg.vocab, size=(B, S)).astype(np.int64)
    mask = np.ones((B, S), np.int64)
    mask[1, 20:] = 0
    from inferc_b200 import structs
    ref = oracle.port().encoder_forward(structs.encoder_struct(cfg, w), ids, mask, 2)
    p = plans.EncoderPlan(cfg, w, max_batch=4, max_seq=64)
    for _ in range(2):
        got = p.run_host(ids, mask)
        np.testing.assert_allclose(got, ref, atol=LOGIT_TOL, rtol=1e-4)
    from inferc_b200 import lib
    assert lib.load().inferc_dev_encoder_range_fallbacks(p._h) == 2


def test_encoder_errors(full_encoder, enc_gold):
    ids = enc_gold["c0_ids"].copy()
    ids[0, 5] = 10 ** 6  # Gather index out of range (embedding.cc:63-65)
    with pytest.raises(InfercError, match="RANGE"):
        full_encoder.run_host(ids, enc_gold["c0_mask"])
    # The plan stays usable after the error.
    got = full_encoder.run_host(enc_gold["c0_ids"], enc_gold["c0_mask"])
    np.testing.assert_allclose(got, enc_gold["c0_logits"], atol=LOGIT_TOL)
    with pytest.raises(InfercError, match="INVALID"):
        full_encoder.run_host(np.zeros((9, 128), np.int64), np.ones((9, 128), np.int64))


def test_decode_small_config_tokens(dec_gold):
    cfg = synth.Gpt2Config(**make_golden.SMALL_GPT2)
    p = plans.DecoderPlan(cfg, synth.gpt2_weights(cfg, seed=8), max_len=64)
    toks, _ = p.decode(dec_gold["small_prompt"], len(dec_gold["small_tokens"]))
    np.testing.assert_array_equal(toks, dec_gold["small_tokens"])
    toks2, _ = p.decode(dec_gold["small_prompt"], len(dec_gold["small_tokens"]))
    np.testing.assert_array_equal(toks2, dec_gold["small_tokens"])


def test_decode_gpt2_small_full_config(dec_gold):
    cfg = synth.Gpt2Config()
    p = plans.DecoderPlan(cfg, synth.gpt2_weights(cfg, seed=0), max_len=1024)
    toks, ms = p.decode(dec_gold["c1_prompt"], 128)
    np.testing.assert_array_equal(toks, dec_gold["c1_tokens"])
    assert 0 < ms < 50
    # A different prompt length re-captures the step graph.
    toks8, _ = p.decode(dec_gold["c1_prompt"][:8], 4)
    assert toks8.shape == (4,)
    with pytest.raises(InfercError, match="INVALID"):
        p.decode(np.array([50257], np.int64), 2)
    with pytest.raises(InfercError, match="INVALID"):
        p.decode(dec_gold["c1_prompt"], 1024)
