"""Seeded synthetic models and inputs for inferc's benchmark configurations.

There is no network here for HuggingFace checkpoints or datasets, so every
model is random-init with the architecture the reference benchmarks
(DistilBERT-SST2 for `inferc run`, GPT-2-small for `inferc decode`) and every
input is drawn from a seeded generator with the shapes and value ranges of
those workloads. numpy's PCG64 stream is platform independent, so the same
seed gives the same bytes on every machine.

Weight tensors are named after the fields of InfercEncoderWeights /
InfercGpt2Weights (include/inferc_models.h); per-layer tensors carry a
``.{layer}`` suffix.
"""
from __future__ import annotations

import dataclasses

import numpy as np

FLOAT_MIN = float(np.finfo(np.float32).min)


@dataclasses.dataclass(frozen=True)
class EncoderConfig:
    """DistilBERT-architecture encoder (post-LN, erf GELU, CLS head)."""

    layers: int = 6
    hidden: int = 768
    heads: int = 12
    ffn: int = 3072
    vocab: int = 30522
    max_pos: int = 512
    n_classes: int = 2
    ln_eps: float = 1e-12
    attn_fill: float = FLOAT_MIN


@dataclasses.dataclass(frozen=True)
class Gpt2Config:
    """GPT-2-small (pre-LN, tanh GELU, tied LM head)."""

    layers: int = 12
    hidden: int = 768
    heads: int = 12
    ffn: int = 3072
    vocab: int = 50257
    max_pos: int = 1024
    ln_eps: float = 1e-5


ENCODER_LAYER_FIELDS = ("wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "ln1_g",
                        "ln1_b", "w1", "b1", "w2", "b2", "ln2_g", "ln2_b")
GPT2_LAYER_FIELDS = ("ln1_g", "ln1_b", "attn_w", "attn_b", "proj_w", "proj_b",
                     "ln2_g", "ln2_b", "fc_w", "fc_b", "fcproj_w", "fcproj_b")


def _normal(rng: np.random.Generator, shape, std: float = 0.02) -> np.ndarray:
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)


def encoder_weights(cfg: EncoderConfig, seed: int = 0) -> dict[str, np.ndarray]:
    """Weights N(0, 0.02) (biases included), LayerNorm gamma=1 beta=0."""
    rng = np.random.default_rng(seed)
    H, F = cfg.hidden, cfg.ffn
    ones = np.ones(H, np.float32)
    zeros = np.zeros(H, np.float32)
    w: dict[str, np.ndarray] = {
        "word_emb": _normal(rng, (cfg.vocab, H)),
        "pos_emb": _normal(rng, (cfg.max_pos, H)),
        "emb_ln_g": ones.copy(),
        "emb_ln_b": zeros.copy(),
    }
    for l in range(cfg.layers):
        for name in ("wq", "wk", "wv"):
            w[f"{name}.{l}"] = _normal(rng, (H, H))
            w[f"b{name[1]}.{l}"] = _normal(rng, (H,))
        w[f"wo.{l}"] = _normal(rng, (H, H))
        w[f"bo.{l}"] = _normal(rng, (H,))
        w[f"ln1_g.{l}"] = ones.copy()
        w[f"ln1_b.{l}"] = zeros.copy()
        w[f"w1.{l}"] = _normal(rng, (H, F))
        w[f"b1.{l}"] = _normal(rng, (F,))
        w[f"w2.{l}"] = _normal(rng, (F, H))
        w[f"b2.{l}"] = _normal(rng, (H,))
        w[f"ln2_g.{l}"] = ones.copy()
        w[f"ln2_b.{l}"] = zeros.copy()
    w["pre_w"] = _normal(rng, (H, H))
    w["pre_b"] = _normal(rng, (H,))
    w["cls_w"] = _normal(rng, (cfg.n_classes, H))
    w["cls_b"] = _normal(rng, (cfg.n_classes,))
    return w


def gpt2_weights(cfg: Gpt2Config, seed: int = 0) -> dict[str, np.ndarray]:
    """Weights N(0, 0.02) (biases included), LayerNorm gamma=1 beta=0."""
    rng = np.random.default_rng(seed)
    H, F = cfg.hidden, cfg.ffn
    ones = np.ones(H, np.float32)
    zeros = np.zeros(H, np.float32)
    w: dict[str, np.ndarray] = {
        "wte": _normal(rng, (cfg.vocab, H)),
        "wpe": _normal(rng, (cfg.max_pos, H)),
    }
    for l in range(cfg.layers):
        w[f"ln1_g.{l}"] = ones.copy()
        w[f"ln1_b.{l}"] = zeros.copy()
        w[f"attn_w.{l}"] = _normal(rng, (H, 3 * H))
        w[f"attn_b.{l}"] = _normal(rng, (3 * H,))
        w[f"proj_w.{l}"] = _normal(rng, (H, H))
        w[f"proj_b.{l}"] = _normal(rng, (H,))
        w[f"ln2_g.{l}"] = ones.copy()
        w[f"ln2_b.{l}"] = zeros.copy()
        w[f"fc_w.{l}"] = _normal(rng, (H, F))
        w[f"fc_b.{l}"] = _normal(rng, (F,))
        w[f"fcproj_w.{l}"] = _normal(rng, (F, H))
        w[f"fcproj_b.{l}"] = _normal(rng, (H,))
    w["lnf_g"] = ones.copy()
    w["lnf_b"] = zeros.copy()
    return w


def encoder_inputs(batch: int, seq: int, seed: int = 1, vocab: int = 30522,
                   variable_lengths: bool = False) -> tuple[np.ndarray, np.ndarray]:
    """Token ids and attention mask, int64 [batch, seq].

    ids[:, 0] = 101 ([CLS]), ids[:, last valid] = 102 ([SEP]), the rest
    uniform in [1000, vocab-1]. With variable_lengths, each sequence's valid
    length is uniform in [16, seq] (clamped to seq when seq < 16) and the mask
    is 1 on the valid prefix, 0 after it; padded positions hold id 0.
    """
    rng = np.random.default_rng(seed)
    ids = rng.integers(1000, vocab, size=(batch, seq), dtype=np.int64)
    if variable_lengths:
        lo = min(16, seq)
        lens = rng.integers(lo, seq + 1, size=batch)
    else:
        lens = np.full(batch, seq)
    mask = np.zeros((batch, seq), np.int64)
    for b in range(batch):
        n = int(lens[b])
        mask[b, :n] = 1
        ids[b, n:] = 0
        ids[b, 0] = 101
        ids[b, n - 1] = 102
    return ids, mask


def gpt2_prompt(n: int = 32, seed: int = 2, vocab: int = 50257) -> np.ndarray:
    """Prompt token ids uniform in [0, vocab-1], int64 [n]."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, vocab, size=n, dtype=np.int64)


@dataclasses.dataclass(frozen=True)
class Int4Matrix:
    """One int4 GEMV operand: W [N, K/2] packed bytes, scales [N], x [K]."""

    w: np.ndarray
    scales: np.ndarray
    x: np.ndarray

    @property
    def n(self) -> int:
        return int(self.w.shape[0])

    @property
    def k(self) -> int:
        return int(self.x.shape[0])


def pack_int4(q: np.ndarray) -> np.ndarray:
    """Pack signed int4 values q [N, K] in [-8, 7] into [N, K/2] bytes:
    stored nibble = q + 8, even k in the low nibble, odd k in the high."""
    u = (q.astype(np.int16) + 8).astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def int4_matrix(n: int, k: int, rng: np.random.Generator) -> Int4Matrix:
    q = rng.integers(-8, 8, size=(n, k), dtype=np.int8)
    scales = rng.uniform(0.005, 0.02, size=n).astype(np.float32)
    x = rng.standard_normal(k, dtype=np.float32)
    return Int4Matrix(pack_int4(q), scales, x)


GPT2_INT4_SHAPES = ((768, 2304), (768, 768), (768, 3072), (3072, 768))


def gpt2_int4_set(seed: int = 3, layers: int = 12, hidden: int = 768,
                  vocab: int = 50257) -> list[Int4Matrix]:
    """The int4 GEMV workload at GPT-2-small weight volume: per layer the
    (K, N) matrices 768x2304, 768x768, 768x3072, 3072x768, plus the LM head
    768x50257; each with its own batch-1 activation vector."""
    rng = np.random.default_rng(seed)
    mats = []
    for _ in range(layers):
        for k, n in GPT2_INT4_SHAPES:
            mats.append(int4_matrix(n, k, rng))
    mats.append(int4_matrix(vocab, hidden, rng))
    return mats


def attention_sweep_inputs(batch: int, seq: int, hidden: int = 768, seed: int = 4):
    """QKV + attention sweep case: X N(0,1) [batch, seq, hidden], Wq/Wk/Wv
    N(0,0.02) [hidden, hidden], biases N(0,0.02), per-sequence valid lengths
    uniform in [16, seq]. Returns (x, (wq,bq,wk,bk,wv,bv), lens)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, seq, hidden), dtype=np.float32)
    ws = []
    for _ in range(3):
        ws.append(_normal(rng, (hidden, hidden)))
        ws.append(_normal(rng, (hidden,)))
    lens = rng.integers(min(16, seq), seq + 1, size=batch)
    return x, tuple(ws), lens


def quantize_int4_rowscale(w: np.ndarray, trans: bool = False) -> Int4Matrix:
    """Per-output-row symmetric int4 quantisation, the packer of
    inferc_dev_int4_pack_rowscale restated in numpy (bit-identical): output
    row r is column r of a [K, N] Conv1D weight (row r of an [N, K] weight
    when trans); s_r = max|w| / 7 (1 for an all-zero row), q = clip(rint(w /
    s_r), -8, 7). Returns the packed matrix with x = zeros(K)."""
    rows = np.ascontiguousarray(w if trans else w.T, np.float32)  # [N, K]
    m = np.abs(rows).max(axis=1)
    s = np.where(m > 0, m / np.float32(7), np.float32(1)).astype(np.float32)
    q = np.clip(np.rint(rows / s[:, None]), -8, 7).astype(np.int8)
    return Int4Matrix(pack_int4(q), s, np.zeros(rows.shape[1], np.float32))


def dequantize_int4_rowscale(m: Int4Matrix, trans: bool = False) -> np.ndarray:
    """The fp32 weight an int4 row GEMV applies: s_r * (q - 8) formed in fp32
    (bench/amx/int4_gemv_amx.cc:265-267), back in the source layout."""
    lo = (m.w & 0x0F).astype(np.int16) - 8
    hi = (m.w >> 4).astype(np.int16) - 8
    q = np.empty((m.w.shape[0], 2 * m.w.shape[1]), np.float32)
    q[:, 0::2] = lo
    q[:, 1::2] = hi
    rows = (m.scales[:, None] * q).astype(np.float32)
    return np.ascontiguousarray(rows if trans else rows.T)


def gpt2_weights_int4_dequantized(cfg: Gpt2Config, w: dict) -> dict:
    """The GPT-2 weights the int4 decoder plan computes with: the four layer
    matrices and the tied LM head replaced by their int4 round trip. The
    embedding lookup keeps the fp32 wte, so the LM head is returned
    separately as "lm_head" ([vocab, hidden])."""
    out = dict(w)
    for l in range(cfg.layers):
        for name in ("attn_w", "proj_w", "fc_w", "fcproj_w"):
            k = f"{name}.{l}"
            out[k] = dequantize_int4_rowscale(quantize_int4_rowscale(w[k]))
    out["lm_head"] = dequantize_int4_rowscale(quantize_int4_rowscale(w["wte"], trans=True),
                                              trans=True)
    return out
