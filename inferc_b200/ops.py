"""Host mirror of the reference's kernel API (namespace inferc::rt) over
device tensors.

Each function keeps the reference's name, argument meaning, attribute
defaults and error behaviour (RuntimeError on a dtype / rank / shape
mismatch) and runs the corresponding libinferc_b200 entry point on the
current CUDA stream. torch is used only to own device memory and streams.

Reference signatures (src/kernels/*.h):
  FusedMatMulAddGELU(x, w, bias)                fused_matmul_add_gelu.h:22
  FusedQKVProjection(x, wq, bq, wk, bk, wv, bv) attention.h:34
  FusedAttention(q, k, v, mask_cond, head_dim, fill)   attention.h:24
  LayerNorm(x, scale, bias, eps, normalized_dims)      activation.h:26
  Gemm(a, b, c, alpha, beta, trans_a, trans_b)  matmul.h:19
  MatMul(a, b)                                  matmul.h:17
  Gelu / GeluTanh / Softmax(x, axis)            activation.h:14-24
"""
from __future__ import annotations

import ctypes

import torch

from . import lib as _lib
from .lib import InfercError, Int4Gemv

__all__ = ["FusedMatMulAddGELU", "FusedQKVProjection", "FusedAttention", "LayerNorm", "Gemm",
           "MatMul", "Gelu", "GeluTanh", "Softmax", "Gemv", "Int4GemvRowScale",
           "Int4GemvBatched", "Argmax", "InfercError"]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _f32(name: str, *ts: torch.Tensor) -> None:
    for t in ts:
        if t.dtype != torch.float32:
            raise RuntimeError(f"{name}: float32 only")
        if not t.is_cuda:
            raise RuntimeError(f"{name}: tensors must be on a CUDA device")


def _c(t: torch.Tensor) -> torch.Tensor:
    # Reference kernels call .Contiguous() on their inputs.
    return t.contiguous()


def FusedMatMulAddGELU(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    _f32("FusedMatMulAddGELU", x, w, bias)
    if w.dim() != 2:
        raise RuntimeError("FusedMatMulAddGELU: W must be 2D [K, N]")
    if bias.dim() != 1:
        raise RuntimeError("FusedMatMulAddGELU: bias must be 1D [N]")
    if x.dim() < 2:
        raise RuntimeError("FusedMatMulAddGELU: X must be at least 2D")
    K, N = w.shape
    if x.shape[-1] != K:
        raise RuntimeError("FusedMatMulAddGELU: K mismatch between X and W")
    if bias.shape[0] != N:
        raise RuntimeError("FusedMatMulAddGELU: bias size must equal N")
    x, w, bias = _c(x), _c(w), _c(bias)
    M = x.numel() // K
    y = torch.empty(*x.shape[:-1], N, device=x.device, dtype=torch.float32)
    _lib.check(_lib.load().inferc_dev_fused_matmul_add_gelu(
        x.data_ptr(), w.data_ptr(), bias.data_ptr(), y.data_ptr(), M, K, N, _stream()))
    return y


def FusedQKVProjection(x, wq, bq, wk, bk, wv, bv) -> list[torch.Tensor]:
    _f32("FusedQKV", x, wq, bq, wk, bk, wv, bv)
    K = x.shape[-1]
    N = wq.shape[1]
    for w, b in ((wq, bq), (wk, bk), (wv, bv)):
        if w.dim() != 2 or w.shape != (K, N) or b.shape != (N,):
            raise RuntimeError("FusedQKV: weights must be [K, N] with [N] biases")
    x = _c(x)
    M = x.numel() // K
    outs = [torch.empty(*x.shape[:-1], N, device=x.device) for _ in range(3)]
    args = [_c(t).data_ptr() for t in (wq, bq, wk, bk, wv, bv)]
    _lib.check(_lib.load().inferc_dev_fused_qkv(
        x.data_ptr(), *args, *[o.data_ptr() for o in outs], M, K, N, _stream()))
    return outs


def FusedAttention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   mask_cond: torch.Tensor | None = None, head_dim: int = 64,
                   fill: float = -3.0e38) -> torch.Tensor:
    """mask_cond: bool/uint8, true = masked (score replaced by `fill`),
    broadcastable to [B, nH, S, S]. Defaults follow the executor
    (src/runtime/executor.cc:218-224)."""
    _f32("FusedAttention", q, k, v)
    if q.dim() != 3:
        raise RuntimeError("FusedAttention: expect [B,S,H]")
    B, S, H = q.shape
    if head_dim <= 0 or H % head_dim != 0:
        raise RuntimeError("FusedAttention: H not divisible by head_dim")
    q, k, v = _c(q), _c(k), _c(v)
    out = torch.empty_like(q)
    mp, shp, rank = None, None, 0
    if mask_cond is not None and mask_cond.dim() > 0 and mask_cond.numel() > 0:
        m = _c(mask_cond.to(torch.uint8))
        shape = (ctypes.c_int64 * m.dim())(*m.shape)
        mp, shp, rank = m.data_ptr(), ctypes.cast(shape, ctypes.c_void_p), m.dim()
        keep = (m, shape)  # noqa: F841 - keep alive for the call
    _lib.check(_lib.load().inferc_dev_fused_attention(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), mp, shp, rank, B, S, H, head_dim, fill,
        out.data_ptr(), _stream()))
    return out


def LayerNorm(x: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor, eps: float = 1e-12,
              normalized_dims: int = 1) -> torch.Tensor:
    _f32("LayerNorm", x, scale, bias)
    if normalized_dims < 1 or normalized_dims > x.dim():
        raise RuntimeError("LayerNorm: bad normalized_dims")
    feat = 1
    for d in x.shape[x.dim() - normalized_dims:]:
        feat *= d
    if scale.numel() != feat or bias.numel() != feat:
        raise RuntimeError("LayerNorm: scale/bias size mismatch with feature dim")
    x, scale, bias = _c(x), _c(scale), _c(bias)
    y = torch.empty_like(x)
    _lib.check(_lib.load().inferc_dev_layernorm(x.data_ptr(), scale.data_ptr(), bias.data_ptr(),
                                                y.data_ptr(), x.numel() // feat, feat, eps,
                                                _stream()))
    return y


def Gemm(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor | None = None, alpha: float = 1.0,
         beta: float = 1.0, trans_a: bool = False, trans_b: bool = False) -> torch.Tensor:
    _f32("Gemm", a, b)
    if a.dim() != 2 or b.dim() != 2:
        raise RuntimeError("Gemm: 2D inputs only")
    M, K = (a.shape[1], a.shape[0]) if trans_a else (a.shape[0], a.shape[1])
    Kb, N = (b.shape[1], b.shape[0]) if trans_b else (b.shape[0], b.shape[1])
    if K != Kb:
        raise RuntimeError("Gemm: K mismatch")
    a, b = _c(a), _c(b)
    y = torch.empty(M, N, device=a.device)
    cp, clen = None, 0
    if c is not None:
        _f32("Gemm", c)
        c = _c(c)
        if beta != 0.0 and not (c.numel() == M * N or (c.dim() == 1 and c.shape[0] in (N, 1))):
            raise RuntimeError("Gemm: unsupported C shape for broadcast")
        cp, clen = c.data_ptr(), c.numel()
    _lib.check(_lib.load().inferc_dev_gemm(a.data_ptr(), b.data_ptr(), cp, clen, y.data_ptr(),
                                           M, K, N, alpha, beta, int(trans_a), int(trans_b),
                                           _stream()))
    return y


def MatMul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """2-D (or leading-dims-flattened) MatMul with a 2-D right operand."""
    _f32("MatMul", a, b)
    if b.dim() != 2 or a.dim() < 1:
        raise RuntimeError("MatMul: right operand must be 2D")
    K, N = b.shape
    if a.shape[-1] != K:
        raise RuntimeError("MatMul: inner dim mismatch (K!=K)")
    a, b = _c(a), _c(b)
    M = a.numel() // K
    y = torch.empty(*a.shape[:-1], N, device=a.device)
    _lib.check(_lib.load().inferc_dev_matmul(a.data_ptr(), b.data_ptr(), y.data_ptr(), M, K, N,
                                             _stream()))
    return y


def _unary(name, fn, x):
    _f32(name, x)
    x = _c(x)
    y = torch.empty_like(x)
    _lib.check(getattr(_lib.load(), fn)(x.data_ptr(), y.data_ptr(), x.numel(), _stream()))
    return y


def Gelu(x: torch.Tensor) -> torch.Tensor:
    return _unary("Gelu", "inferc_dev_gelu", x)


def GeluTanh(x: torch.Tensor) -> torch.Tensor:
    return _unary("GeluTanh", "inferc_dev_gelu_tanh", x)


def Softmax(x: torch.Tensor, axis: int = -1) -> torch.Tensor:
    _f32("Softmax", x)
    if axis < 0:
        axis += x.dim()
    if axis < 0 or axis >= x.dim():
        raise RuntimeError("Softmax: axis out of range")
    moved = _c(x.movedim(axis, -1))
    y = torch.empty_like(moved)
    _lib.check(_lib.load().inferc_dev_softmax(moved.data_ptr(), y.data_ptr(),
                                              moved.numel() // moved.shape[-1], moved.shape[-1],
                                              _stream()))
    return y.movedim(-1, axis).contiguous()


ACTS = {None: 0, "gelu": 1, "gelu_tanh": 2, "relu": 3}


def Gemv(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
         resid: torch.Tensor | None = None, act: str | None = None,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """Batch-1 decode GEMV y = act(x W + b + resid), W [K, N]."""
    _f32("Gemv", x, w)
    K, N = w.shape
    y = out if out is not None else torch.empty(N, device=x.device)
    _lib.check(_lib.load().inferc_dev_gemv(
        _c(x).data_ptr(), _c(w).data_ptr(), None if bias is None else _c(bias).data_ptr(),
        None if resid is None else _c(resid).data_ptr(), y.data_ptr(), K, N, ACTS[act],
        _stream()))
    return y


def Int4GemvRowScale(w: torch.Tensor, scales: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """w: uint8 [N, K/2] packed nibbles; scales fp32 [N]; x fp32 [K]."""
    if w.dtype != torch.uint8:
        raise RuntimeError("Int4Gemv: weights must be packed uint8")
    _f32("Int4Gemv", scales, x)
    N, K = w.shape[0], x.shape[0]
    if w.shape[1] * 2 != K:
        raise RuntimeError("Int4Gemv: W must be [N, K/2]")
    y = torch.empty(N, device=x.device)
    _lib.check(_lib.load().inferc_dev_gemv_int4_rowscale(
        _c(w).data_ptr(), _c(scales).data_ptr(), _c(x).data_ptr(), y.data_ptr(), N, K,
        _stream()))
    return y


def Int4GemvBatched(mats: list[tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]]):
    """mats: list of (w_packed, scales, x, y_out); one launch per K class."""
    arr = (Int4Gemv * len(mats))()
    for i, (w, s, x, y) in enumerate(mats):
        arr[i] = Int4Gemv(w.data_ptr(), s.data_ptr(), x.data_ptr(), y.data_ptr(), w.shape[0],
                          x.shape[0])
    _lib.check(_lib.load().inferc_dev_gemv_int4_batched(arr, len(mats), _stream()))


def Argmax(x: torch.Tensor) -> torch.Tensor:
    """Index of the first maximum (int64 scalar tensor on the device)."""
    _f32("Argmax", x)
    out = torch.empty((), dtype=torch.int64, device=x.device)
    _lib.check(_lib.load().inferc_dev_argmax(_c(x).data_ptr(), x.numel(), out.data_ptr(),
                                             _stream()))
    return out
