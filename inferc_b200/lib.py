"""Loads libinferc_b200.so (built in-tree by inferc_b200/build.py) and
declares the ctypes signatures of every entry point in include/inferc_dev.h.

There is no CPU fallback: if the library is missing, `load()` raises.
"""
from __future__ import annotations

import ctypes
import os

from . import structs

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libinferc_b200.so")

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t


class Int4Gemv(ctypes.Structure):
    """Mirror of InfercInt4Gemv."""

    _fields_ = [("w", _p), ("scales", _p), ("x", _p), ("y", _p), ("n", _i64), ("k", _i64)]


# name -> (argtypes, restype); restype None means void.
SIGNATURES: dict[str, tuple[list, object]] = {
    "inferc_dev_last_error_string": ([], ctypes.c_char_p),
    "inferc_dev_version": ([], ctypes.c_char_p),
    "inferc_dev_alloc": ([ctypes.POINTER(_p), _sz], _i),
    "inferc_dev_free": ([_p], _i),
    "inferc_dev_memcpy_h2d": ([_p, _p, _sz, _p], _i),
    "inferc_dev_memcpy_d2h": ([_p, _p, _sz, _p], _i),
    "inferc_dev_stream_synchronize": ([_p], _i),
    "inferc_dev_selftest_wait_timeout": ([_i, _i64, _p], _i),
    "inferc_dev_weight_cache_evict": ([_p], _i),
    "inferc_dev_weight_cache_clear": ([], _i),
    "inferc_dev_weight_cache_bytes": ([], _i64),
    "inferc_dev_layernorm": ([_p, _p, _p, _p, _i64, _i64, _f, _p], _i),
    "inferc_dev_fused_matmul_add_gelu": ([_p, _p, _p, _p, _i64, _i64, _i64, _p], _i),
    "inferc_dev_fused_qkv": ([_p] * 10 + [_i64] * 3 + [_p], _i),
    "inferc_dev_fused_attention": ([_p, _p, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _f, _p, _p],
                                   _i),
    "inferc_dev_gemm": ([_p, _p, _p, _i64, _p, _i64, _i64, _i64, _f, _f, _i, _i, _p], _i),
    "inferc_dev_matmul": ([_p, _p, _p, _i64, _i64, _i64, _p], _i),
    "inferc_dev_gelu": ([_p, _p, _i64, _p], _i),
    "inferc_dev_gelu_tanh": ([_p, _p, _i64, _p], _i),
    "inferc_dev_softmax": ([_p, _p, _i64, _i64, _p], _i),
    "inferc_dev_tf32_split": ([_p, _p, _p, _i64, _p], _i),
    "inferc_dev_gemm_tf32x3": ([_p, _i64, _p, _p, _i64, _p, _p, _i64, _p, _i64, _i64, _i64, _i64,
                                _i, _p], _i),
    "inferc_dev_f16_kp": ([_i64], _i64),
    "inferc_dev_f16_split": ([_p, _i64, _i64, _i64, _p, _p, _p, _p], _i),
    "inferc_dev_gemm_f16s": ([_p, _i64, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i,
                              _p], _i),
    "inferc_dev_f16_split_rows": ([_p, _i64, _i64, _i64, _p, _p, _i64, _p], _i),
    "inferc_dev_gemm_f16s_planes": ([_p, _p, _i64, _p, _p, _p, _p, _p, _i64, _p, _p, _p, _i64,
                                     _i64, _i64, _i64, _i, _p], _i),
    "inferc_dev_fused_attention_planes": ([_p] * 6 + [_i64, _p, _i64, _i64, _i64, _f, _p, _p],
                                          _i),
    "inferc_dev_qkv_attention_f16": ([_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _f, _p, _p,
                                      _p], _i),
    "inferc_dev_qkv_attention": ([_p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _f, _p, _p, _p],
                                 _i),
    "inferc_dev_gemv": ([_p, _p, _p, _p, _p, _i64, _i64, _i, _p], _i),
    "inferc_dev_gemv_noalloc": ([_p, _p, _p, _p, _p, _i64, _i64, _i, _p], _i),
    "inferc_dev_gemv_int4_rowscale": ([_p, _p, _p, _p, _i64, _i64, _p], _i),
    "inferc_dev_gemv_int4_batched": ([ctypes.POINTER(Int4Gemv), _i, _p], _i),
    "inferc_dev_argmax": ([_p, _i64, _p, _p], _i),
    "inferc_dev_kv_append": ([_p, _p, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _p], _i),
    "inferc_dev_decode_attention": ([_p, _p, _p, _p, _i64, _i64, _i64, _i64, _p], _i),
    "inferc_dev_graph_describe": ([_p, _sz, _p, _sz, ctypes.POINTER(_sz)], _i),
    "inferc_dev_graph_load": ([_p, _sz, ctypes.POINTER(_p)], _i),
    "inferc_dev_graph_set_input": ([_p, ctypes.c_char_p, _i, _p, _i, _p, _i, _p], _i),
    "inferc_dev_graph_run": ([_p, _p], _i),
    "inferc_dev_graph_output": ([_p, ctypes.c_char_p, ctypes.POINTER(_i), _p, ctypes.POINTER(_i),
                                 ctypes.POINTER(_p)], _i),
    "inferc_dev_graph_destroy": ([_p], None),
    "inferc_dev_encoder_create": ([ctypes.POINTER(structs.EncoderWeights), _i64, _i64,
                                   ctypes.POINTER(_p)], _i),
    "inferc_dev_encoder_run": ([_p, _p, _p, _i64, _i64, _p, _p], _i),
    "inferc_dev_encoder_run_host": ([_p, _p, _p, _i64, _i64, _p], _i),
    "inferc_dev_encoder_range_fallbacks": ([_p], _i64),
    "inferc_dev_encoder_destroy": ([_p], None),
    "inferc_dev_decoder_create": ([ctypes.POINTER(structs.Gpt2Weights), _i64,
                                   ctypes.POINTER(_p)], _i),
    "inferc_dev_decoder_create_int4": ([ctypes.POINTER(structs.Gpt2Weights), _i64,
                                        ctypes.POINTER(_p)], _i),
    "inferc_dev_int4_pack_rowscale": ([_p, _i64, _i64, _i64, _i, _p, _p, _p], _i),
    "inferc_dev_decode": ([_p, _p, _i64, _i64, _p, ctypes.POINTER(ctypes.c_double)], _i),
    "inferc_dev_decoder_logits": ([_p], _p),
    "inferc_dev_decoder_destroy": ([_p], None),
}

ERRORS = {1: "INVALID", 2: "CUDA", 3: "OOM", 4: "TIMEOUT", 5: "RANGE"}


class InfercError(RuntimeError):
    """A non-zero status from the C ABI (the reference throws
    std::runtime_error at the same points)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{ERRORS.get(code, code)}] {msg}")
        self.code = code


_lib = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m inferc_b200.build`")
    lib = ctypes.CDLL(path)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != 0:
        msg = load().inferc_dev_last_error_string().decode()
        raise InfercError(rc, msg)
