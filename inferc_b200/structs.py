"""ctypes mirrors of the C weight tables in include/inferc_models.h, plus
helpers that fill them from a dict of named arrays (numpy for host pointers,
torch CUDA tensors for device pointers)."""
from __future__ import annotations

import ctypes

MAX_LAYERS = 48
_P = ctypes.c_void_p
_PL = _P * MAX_LAYERS


class EncoderWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("layers", "hidden", "heads", "ffn", "vocab", "max_pos", "n_classes")] + [
        ("ln_eps", ctypes.c_float), ("attn_fill", ctypes.c_float),
        ("word_emb", _P), ("pos_emb", _P), ("emb_ln_g", _P), ("emb_ln_b", _P),
    ] + [(n, _PL) for n in ("wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "ln1_g", "ln1_b",
                            "w1", "b1", "w2", "b2", "ln2_g", "ln2_b")] + [
        ("pre_w", _P), ("pre_b", _P), ("cls_w", _P), ("cls_b", _P)]


class Gpt2Weights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("layers", "hidden", "heads", "ffn", "vocab", "max_pos")] + [
        ("ln_eps", ctypes.c_float), ("wte", _P), ("wpe", _P),
    ] + [(n, _PL) for n in ("ln1_g", "ln1_b", "attn_w", "attn_b", "proj_w", "proj_b",
                            "ln2_g", "ln2_b", "fc_w", "fc_b", "fcproj_w", "fcproj_b")] + [
        ("lnf_g", _P), ("lnf_b", _P)]


def _addr(a) -> int:
    if hasattr(a, "data_ptr"):  # torch tensor
        assert a.is_contiguous()
        return a.data_ptr()
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _fill(struct, cfg, tensors, layer_fields, scalars):
    if cfg.layers > MAX_LAYERS:
        raise ValueError(f"layers={cfg.layers} exceeds {MAX_LAYERS}")
    s = struct()
    for name in scalars:
        setattr(s, name, getattr(cfg, name))
    for name, _ in struct._fields_:
        if name in scalars:
            continue
        if name in layer_fields:
            arr = getattr(s, name)
            for l in range(cfg.layers):
                arr[l] = _addr(tensors[f"{name}.{l}"])
        else:
            setattr(s, name, _addr(tensors[name]))
    s._keep = tensors  # the table holds raw addresses: keep the arrays alive with it
    return s


def encoder_struct(cfg, tensors) -> EncoderWeights:
    from .synth import ENCODER_LAYER_FIELDS
    return _fill(EncoderWeights, cfg, tensors, ENCODER_LAYER_FIELDS,
                 ("layers", "hidden", "heads", "ffn", "vocab", "max_pos", "n_classes",
                  "ln_eps", "attn_fill"))


def gpt2_struct(cfg, tensors) -> Gpt2Weights:
    from .synth import GPT2_LAYER_FIELDS
    return _fill(Gpt2Weights, cfg, tensors, GPT2_LAYER_FIELDS,
                 ("layers", "hidden", "heads", "ffn", "vocab", "max_pos", "ln_eps"))
