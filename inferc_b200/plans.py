"""Python handles for the prepared device plans of libinferc_b200:

  EncoderPlan - the DistilBERT-architecture encoder plan run by `inferc run`
                (src/cli/main.cpp:324-420): ids/mask -> logits.
  DecoderPlan - GPT-2 greedy decode with a device KV cache, `inferc decode`
                (src/cli/main.cpp:700-945): prompt -> generated token ids.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import lib as _lib
from . import structs


class EncoderPlan:
    def __init__(self, cfg, weights: dict, max_batch: int, max_seq: int):
        """weights: host numpy arrays named as in inferc_b200.synth (copied to
        the current CUDA device once)."""
        self.cfg = cfg
        self._w = structs.encoder_struct(cfg, weights)
        h = ctypes.c_void_p()
        L = _lib.load()
        _lib.check(L.inferc_dev_encoder_create(ctypes.byref(self._w), max_batch, max_seq,
                                               ctypes.byref(h)))
        self._h = h
        self.max_batch, self.max_seq = max_batch, max_seq

    def run_host(self, ids: np.ndarray, mask: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int64)
        mask = np.ascontiguousarray(mask, np.int64)
        B, S = ids.shape
        logits = np.empty((B, self.cfg.n_classes), np.float32)
        _lib.check(_lib.load().inferc_dev_encoder_run_host(
            self._h, ids.ctypes.data, mask.ctypes.data, B, S, logits.ctypes.data))
        return logits

    def run(self, ids, mask, logits, stream: int = 0) -> None:
        """ids / mask: int64 device tensors [B,S]; logits: fp32 device [B,C]."""
        B, S = ids.shape
        _lib.check(_lib.load().inferc_dev_encoder_run(
            self._h, ids.data_ptr(), mask.data_ptr(), B, S, logits.data_ptr(), stream))

    def close(self) -> None:
        if self._h:
            _lib.load().inferc_dev_encoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DecoderPlan:
    def __init__(self, cfg, weights: dict, max_len: int = 1024, int4: bool = False):
        """int4: the weight-only int4 decoder (inferc_dev_decoder_create_int4)."""
        self.cfg = cfg
        self._w = structs.gpt2_struct(cfg, weights)
        h = ctypes.c_void_p()
        L = _lib.load()
        create = L.inferc_dev_decoder_create_int4 if int4 else L.inferc_dev_decoder_create
        _lib.check(create(ctypes.byref(self._w), max_len, ctypes.byref(h)))
        self._h = h
        self.max_len = max_len

    def decode(self, prompt: np.ndarray, max_tokens: int) -> tuple[np.ndarray, float]:
        """Returns (token ids [max_tokens], mean device ms per single-token step)."""
        prompt = np.ascontiguousarray(prompt, np.int64)
        toks = np.empty(max_tokens, np.int64)
        ms = ctypes.c_double(0.0)
        _lib.check(_lib.load().inferc_dev_decode(self._h, prompt.ctypes.data, prompt.size,
                                                 max_tokens, toks.ctypes.data, ctypes.byref(ms)))
        return toks, ms.value

    def logits_ptr(self) -> int:
        return _lib.load().inferc_dev_decoder_logits(self._h)

    def close(self) -> None:
        if self._h:
            _lib.load().inferc_dev_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
