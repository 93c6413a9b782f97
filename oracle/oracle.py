"""ctypes bindings for the two CPU oracles. TEST INFRASTRUCTURE ONLY: imported
by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs, never by
the product package.

  port() -> oracle/_build/liborc_port.so  (C restatement, inferc_oracle.c)
  ref()  -> oracle/_ref/libinferc_ref.so  (the reference's own kernel sources,
            built by oracle/Makefile; present only where the reference checkout
            (INFERC_REF_ROOT, or the Makefile's REF) was available at build time, None otherwise)
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "_build", "liborc_port.so")
REF_SO = os.path.join(HERE, "_ref", "libinferc_ref.so")

_f = ctypes.c_float
_i64 = ctypes.c_int64
_p = ctypes.c_void_p
_i = ctypes.c_int


# Root of the reference checkout whose kernel sources `make ref` compiles:
# INFERC_REF_ROOT when set, else the Makefile's default REF.
def _ref_root() -> str:
    env = os.environ.get("INFERC_REF_ROOT")
    if env:
        return env
    with open(os.path.join(HERE, "Makefile")) as f:
        for line in f:
            if line.startswith("REF ?="):
                return line.split("=", 1)[1].strip()
    return ""


def build(with_ref: bool = True) -> None:
    targets = ["port"]
    root = _ref_root()
    extra = [f"REF={root}"] if root else []
    if with_ref and root and os.path.isdir(os.path.join(root, "src")):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE] + extra + targets, check=True)


def ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data


class _Lib:
    def __init__(self, path: str, prefix: str):
        self.lib = ctypes.CDLL(path)
        self.prefix = prefix

    def fn(self, name, argtypes, restype=_i):
        f = getattr(self.lib, self.prefix + name)
        f.argtypes = argtypes
        f.restype = restype
        return f


_port = None
_ref = None


def port():
    """The C restatement; builds it on first use if missing."""
    global _port
    if _port is None:
        if not os.path.exists(PORT_SO):
            build(with_ref=False)
        _port = Port(PORT_SO)
    return _port


def ref():
    """The reference's own kernels, or None when they were not built."""
    global _ref
    if _ref is None and os.path.exists(REF_SO):
        _ref = Ref(REF_SO)
    return _ref


class _Ops:
    """Numpy-level wrappers shared by the port and the reference builds."""

    kind = ""

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(f"{self.kind} oracle call failed ({rc})")

    def layernorm(self, x, g, b, eps):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        feat = x.shape[-1]
        self._check(self._ln(ptr(x), ptr(g), ptr(b), ptr(y), x.size // feat, feat, eps))
        return y

    def fused_matmul_add_gelu(self, x, w, b):
        x = np.ascontiguousarray(x, np.float32)
        K, N = w.shape
        M = x.size // K
        y = np.empty(x.shape[:-1] + (N,), np.float32)
        self._check(self._mmg(ptr(x), ptr(w), ptr(b), ptr(y), M, K, N))
        return y

    def fused_qkv(self, x, wq, bq, wk, bk, wv, bv):
        x = np.ascontiguousarray(x, np.float32)
        K, N = wq.shape
        M = x.size // K
        outs = [np.empty(x.shape[:-1] + (N,), np.float32) for _ in range(3)]
        self._check(self._qkv(ptr(x), ptr(wq), ptr(bq), ptr(wk), ptr(bk), ptr(wv), ptr(bv),
                              *[ptr(o) for o in outs], M, K, N))
        return outs

    def fused_attention(self, q, k, v, mask, head_dim, fill):
        B, S, H = q.shape
        out = np.empty_like(q)
        if mask is None:
            mp, shp, rank = None, None, 0
        else:
            mask = np.ascontiguousarray(mask, np.uint8)
            shp_arr = np.array(mask.shape, np.int64)
            mp, shp, rank = ptr(mask), ptr(shp_arr), mask.ndim
        self._check(self._attn(ptr(q), ptr(k), ptr(v), mp, shp, rank, B, S, H, head_dim,
                               fill, ptr(out)))
        return out

    def gemm(self, a, b, c, alpha=1.0, beta=1.0, trans_a=False, trans_b=False):
        M = a.shape[1] if trans_a else a.shape[0]
        K = a.shape[0] if trans_a else a.shape[1]
        N = b.shape[0] if trans_b else b.shape[1]
        y = np.empty((M, N), np.float32)
        clen = 0 if c is None else c.size
        self._check(self._gemm(ptr(a), ptr(b), ptr(c), clen, ptr(y), M, K, N, alpha, beta,
                               int(trans_a), int(trans_b)))
        return y

    def gelu_tanh(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self._check(self._gt(ptr(x), ptr(y), x.size))
        return y

    def gelu(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self._check(self._ge(ptr(x), ptr(y), x.size))
        return y

    def softmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self._check(self._sm(ptr(x), ptr(y), x.size // x.shape[-1], x.shape[-1]))
        return y

    def encoder_forward(self, wstruct, ids, mask, n_classes):
        B, S = ids.shape
        logits = np.empty((B, n_classes), np.float32)
        self._check(self._enc(ctypes.byref(wstruct), ptr(ids), ptr(mask), B, S, ptr(logits)))
        return logits


_SIG = {
    "layernorm": [_p, _p, _p, _p, _i64, _i64, _f],
    "fused_matmul_add_gelu": [_p, _p, _p, _p, _i64, _i64, _i64],
    "fused_qkv": [_p] * 10 + [_i64] * 3,
    "fused_attention": [_p, _p, _p, _p, _p, _i, _i64, _i64, _i64, _i64, _f, _p],
    "gemm": [_p, _p, _p, _i64, _p, _i64, _i64, _i64, _f, _f, _i, _i],
    "gelu_tanh": [_p, _p, _i64],
    "gelu": [_p, _p, _i64],
    "softmax": [_p, _p, _i64, _i64],
    "encoder_forward": [_p, _p, _p, _i64, _i64, _p],
}


def _bind(obj, lib, void_names=()):
    names = {"layernorm": "_ln", "fused_matmul_add_gelu": "_mmg", "fused_qkv": "_qkv",
             "fused_attention": "_attn", "gemm": "_gemm", "gelu_tanh": "_gt", "gelu": "_ge",
             "softmax": "_sm", "encoder_forward": "_enc"}
    for cname, attr in names.items():
        f = lib.fn(cname, _SIG[cname], None if cname in void_names else _i)
        if cname in void_names:
            g = f
            f = (lambda g: (lambda *a: (g(*a), 0)[1]))(g)
        setattr(obj, attr, f)


class Port(_Ops):
    kind = "port"

    def __init__(self, path):
        self._l = _Lib(path, "orc_")
        _bind(self, self._l, void_names=("layernorm", "fused_matmul_add_gelu", "fused_qkv",
                                         "fused_attention", "gelu_tanh", "gelu", "softmax"))
        self._int4 = self._l.fn("int4_gemv_rowscale", [_p, _p, _p, _p, _i64, _i64], None)
        self._int4t = self._l.fn("int4_gemv", [_p, _f, _p, _p, _i64, _i64], None)
        self._dec = self._l.fn("gpt2_decode", [_p, _p, _i64, _i64, _p, _p])
        self._declm = self._l.fn("gpt2_decode_lm", [_p, _p, _p, _i64, _i64, _p, _p])
        self._argmax = self._l.fn("argmax", [_p, _i64], _i64)

    def int4_gemv_rowscale(self, w, scales, x):
        N = w.shape[0]
        K = x.shape[0]
        y = np.empty(N, np.float32)
        self._int4(ptr(w), ptr(scales), ptr(x), ptr(y), N, K)
        return y

    def int4_gemv(self, w, scale, x):
        N = w.shape[0]
        K = x.shape[0]
        y = np.empty(N, np.float32)
        self._int4t(ptr(w), scale, ptr(x), ptr(y), N, K)
        return y

    def argmax(self, x):
        x = np.ascontiguousarray(x, np.float32)
        return int(self._argmax(ptr(x), x.size))

    def gpt2_decode(self, wstruct, prompt, max_tokens):
        prompt = np.ascontiguousarray(prompt, np.int64)
        toks = np.empty(max_tokens, np.int64)
        margins = np.empty(max_tokens, np.float32)
        self._check(self._dec(ctypes.byref(wstruct), ptr(prompt), prompt.size, max_tokens,
                              ptr(toks), ptr(margins)))
        return toks, margins

    def gpt2_decode_lm(self, wstruct, lm_head, prompt, max_tokens):
        """Greedy decode with a separate LM head [vocab, hidden]."""
        prompt = np.ascontiguousarray(prompt, np.int64)
        lm_head = np.ascontiguousarray(lm_head, np.float32)
        toks = np.empty(max_tokens, np.int64)
        margins = np.empty(max_tokens, np.float32)
        self._check(self._declm(ctypes.byref(wstruct), ptr(lm_head), ptr(prompt), prompt.size,
                                max_tokens, ptr(toks), ptr(margins)))
        return toks, margins


class Ref(_Ops):
    kind = "reference"

    def __init__(self, path):
        self._l = _Lib(path, "ref_")
        _bind(self, self._l)
        self._dec = self._l.fn("gpt2_decode", [_p, _p, _i64, _i64, _p, _p, _p])
        self._declm = self._l.fn("gpt2_decode_lm", [_p, _p, _p, _i64, _i64, _p, _p, _p])
        self._err = self._l.fn("last_error", [], ctypes.c_char_p)

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError("reference oracle: " + self._err().decode())

    def gpt2_decode(self, wstruct, prompt, max_tokens):
        """Returns (tokens, margins, mean step ms)."""
        prompt = np.ascontiguousarray(prompt, np.int64)
        toks = np.empty(max_tokens, np.int64)
        margins = np.empty(max_tokens, np.float32)
        ms = ctypes.c_double(0.0)
        self._check(self._dec(ctypes.byref(wstruct), ptr(prompt), prompt.size, max_tokens,
                              ptr(toks), ptr(margins), ctypes.byref(ms)))
        return toks, margins, ms.value

    def gpt2_decode_lm(self, wstruct, lm_head, prompt, max_tokens):
        """Greedy decode with a separate LM head [vocab, hidden]; returns
        (tokens, margins, mean step ms)."""
        prompt = np.ascontiguousarray(prompt, np.int64)
        lm_head = np.ascontiguousarray(lm_head, np.float32)
        toks = np.empty(max_tokens, np.int64)
        margins = np.empty(max_tokens, np.float32)
        ms = ctypes.c_double(0.0)
        self._check(self._declm(ctypes.byref(wstruct), ptr(lm_head), ptr(prompt), prompt.size,
                                max_tokens, ptr(toks), ptr(margins), ctypes.byref(ms)))
        return toks, margins, ms.value
