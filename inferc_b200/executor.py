"""Host handle of the device executor (inferc_dev_graph_* in
include/inferc_dev.h): runs an optimized inferc plan - ONNX bytes - node by
node on the GPU, the device counterpart of the reference's `inferc run`
(Executor::Run, src/runtime/executor.cc:98-366) and of `inferc decode`'s
prefill + with-past loop (CmdDecode, src/cli/main.cpp:700-945).
"""
from __future__ import annotations

import ctypes
import json
import time

import numpy as np

from . import lib as _lib

_NP = {1: np.float32, 2: np.uint8, 6: np.int32, 7: np.int64, 9: np.bool_}
_CODE = {np.dtype(v): k for k, v in _NP.items()}


def describe(model: bytes) -> dict:
    """Parses the model on the host only (no device) and returns its summary:
    node count, op histogram, opsets, inputs, outputs."""
    L = _lib.load()
    need = ctypes.c_size_t(0)
    _lib.check(L.inferc_dev_graph_describe(model, len(model), None, 0, ctypes.byref(need)))
    buf = ctypes.create_string_buffer(need.value)
    _lib.check(L.inferc_dev_graph_describe(model, len(model), buf, need.value, None))
    return json.loads(buf.value.decode())


class Graph:
    """One loaded plan on the current CUDA device."""

    def __init__(self, model: bytes):
        L = _lib.load()
        self._model = model
        h = ctypes.c_void_p()
        _lib.check(L.inferc_dev_graph_load(model, len(model), ctypes.byref(h)))
        self._h = h

    def set_input(self, name: str, value, stream: int = 0) -> None:
        """value: a numpy array (copied from host) or a CUDA torch tensor
        (copied device to device on `stream`)."""
        L = _lib.load()
        if isinstance(value, np.generic):
            value = np.asarray(value)
        if isinstance(value, np.ndarray):
            a = np.ascontiguousarray(value)
            shape = (ctypes.c_int64 * max(a.ndim, 1))(*a.shape)
            _lib.check(L.inferc_dev_graph_set_input(self._h, name.encode(), _CODE[a.dtype], shape,
                                                    a.ndim, a.ctypes.data, 0, stream))
        else:
            import torch
            t = value.contiguous()
            code = {torch.float32: 1, torch.int64: 7, torch.int32: 6, torch.bool: 9,
                    torch.uint8: 2}[t.dtype]
            shape = (ctypes.c_int64 * max(t.dim(), 1))(*t.shape)
            _lib.check(L.inferc_dev_graph_set_input(self._h, name.encode(), code, shape, t.dim(),
                                                    t.data_ptr(), 1, stream))

    def run(self, stream: int = 0) -> None:
        _lib.check(_lib.load().inferc_dev_graph_run(self._h, stream))

    def output_info(self, name: str) -> tuple[int, tuple, int]:
        """(ONNX dtype code, shape, device address) of an output of the last run."""
        L = _lib.load()
        dt, rank = ctypes.c_int(0), ctypes.c_int(0)
        shape = (ctypes.c_int64 * 8)()
        ptr = ctypes.c_void_p()
        _lib.check(L.inferc_dev_graph_output(self._h, name.encode(), ctypes.byref(dt), shape,
                                             ctypes.byref(rank), ctypes.byref(ptr)))
        return dt.value, tuple(shape[: rank.value]), ptr.value

    def output(self, name: str) -> np.ndarray:
        dt, shape, ptr = self.output_info(name)
        out = np.empty(shape, _NP[dt])
        if out.nbytes:
            _lib.check(_lib.load().inferc_dev_memcpy_d2h(out.ctypes.data, ptr, out.nbytes, None))
            _lib.check(_lib.load().inferc_dev_stream_synchronize(None))
        return out

    def run_host(self, inputs: dict, outputs: list[str]) -> dict:
        for k, v in inputs.items():
            self.set_input(k, v)
        self.run()
        return {k: self.output(k) for k in outputs}

    def close(self) -> None:
        if self._h:
            _lib.load().inferc_dev_graph_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def greedy_decode(prefill: Graph, step: Graph, n_layers: int, prompt: np.ndarray,
                  max_tokens: int) -> tuple[np.ndarray, float]:
    """`inferc decode` over two loaded plans (src/cli/main.cpp:790-889): the
    prefill graph on the prompt, the first token = argmax of the last logits
    row (first maximum wins, on the device), then max_tokens-1 runs of the
    with-past graph, each fed the previous step's present.* tensors as
    past_key_values.* (copied on the device) and the new token. Returns the
    token ids and the mean wall-clock ms per single-token step, as the
    reference reports it."""
    L = _lib.load()
    prompt = np.ascontiguousarray(prompt, np.int64).reshape(1, -1)
    n = prompt.shape[1]
    tok_dev = ctypes.c_void_p()
    _lib.check(L.inferc_dev_alloc(ctypes.byref(tok_dev), 8))
    try:
        prefill.set_input("input_ids", prompt)
        prefill.set_input("attention_mask", np.ones((1, n), np.int64))
        prefill.run()
        toks = []

        def argmax_row(g: Graph, row: int) -> int:
            dt, shape, ptr = g.output_info("logits")
            vocab = shape[-1]
            _lib.check(L.inferc_dev_argmax(ptr + row * vocab * 4, vocab, tok_dev, None))
            t = np.empty(1, np.int64)
            _lib.check(L.inferc_dev_memcpy_d2h(t.ctypes.data, tok_dev, 8, None))
            _lib.check(L.inferc_dev_stream_synchronize(None))
            return int(t[0])

        toks.append(argmax_row(prefill, n - 1))
        src = prefill
        times = []
        for s in range(1, max_tokens):
            t0 = time.perf_counter()
            for l in range(n_layers):
                for kind in ("key", "value"):
                    dt, shape, ptr = src.output_info(f"present.{l}.{kind}")
                    sh = (ctypes.c_int64 * 4)(*shape)
                    _lib.check(L.inferc_dev_graph_set_input(
                        step._h, f"past_key_values.{l}.{kind}".encode(), dt, sh, len(shape),
                        ptr, 1, None))
            step.set_input("input_ids", np.array([[toks[-1]]], np.int64))
            step.set_input("attention_mask", np.ones((1, n + s), np.int64))
            step.run()
            toks.append(argmax_row(step, 0))
            times.append(time.perf_counter() - t0)
            src = step
        return np.array(toks, np.int64), (1e3 * float(np.mean(times)) if times else 0.0)
    finally:
        _lib.check(L.inferc_dev_free(tok_dev))
