"""Device tensor operations of the encoder, mirroring fiber/ai's ``tensor``.

Each function has the name, argument meaning and error behaviour of the
reference's operation and runs it through libfgemma's C ABI on CUDA
tensors (torch is used here only to hold device memory and streams):

- ``MatMul`` / ``MatMulFused`` / ``Fused``: tensor/matmul.go:19,
  tensor/matmul_fused.go:17-96 (epilogue order bias → RowScale → Act → Mul
  → Residual);
- ``RowSumSquares``: tensor/matmul_fused.go:125-143;
- ``RMSNorm``: tensor/attention.go:292-337;
- ``RoPE``: tensor/rope.go:20-87;
- ``AttentionScaled`` with the padding / window masks the encoder builds
  (``PaddingMask`` attention.go:33-42, ``WindowMask`` attention.go:97-107).

Shape errors raise ``TensorError`` with the reference's operation name,
where the reference panics with ``*tensor.Error`` (tensor/errors.go:13).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import ACT_GELU, ACT_NONE, ACT_RELU, PREC_SPLIT, PREC_SPLIT_TF32, PREC_TF32  # noqa: F401

NoAct = ACT_NONE
ReLUAct = ACT_RELU
GELUAct = ACT_GELU


class TensorError(ValueError):
    """A shape or argument error, raised where the reference panics."""

    def __init__(self, op: str, msg: str):
        super().__init__(f"tensor.{op}: {msg}")
        self.op = op


def _fail(op: str, msg: str):
    raise TensorError(op, msg)


def _stream(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _f32_cuda(op: str, name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor) or t.dtype != torch.float32 or not t.is_cuda:
        _fail(op, f"{name} must be a float32 CUDA tensor")


@dataclass
class Fused:
    """Epilogue of MatMulFused (tensor/matmul_fused.go:17-23)."""

    Bias: Optional[torch.Tensor] = None
    Act: int = NoAct
    Mul: Optional[torch.Tensor] = None
    RowScale: Optional[torch.Tensor] = None
    Residual: Optional[torch.Tensor] = None


def MatMulFused(x: torch.Tensor, w: torch.Tensor, f: Fused = Fused(),
                precision: int = PREC_SPLIT) -> torch.Tensor:
    """epilogue(x · w) for 2-D x [m×k] and w [k×n] (matmul_fused.go:40-96).

    ``w`` may be a transposed view of an [n×k] row-major matrix (``W.t()``),
    which is consumed without a copy, like the reference's ``w.T()``.
    """
    op = "MatMulFused"
    _f32_cuda(op, "x", x)
    _f32_cuda(op, "w", w)
    if x.dim() != 2 or w.dim() != 2:
        _fail(op, f"expected 2-D operands, got {list(x.shape)} and {list(w.shape)}")
    m, k = x.shape
    n = w.shape[1]
    if k != w.shape[0]:
        _fail(op, f"shape mismatch {list(x.shape)} · {list(w.shape)}")
    if f.Bias is not None and f.Bias.numel() != n:
        _fail(op, f"bias has {f.Bias.numel()} elements for {n} columns")
    if f.RowScale is not None and f.RowScale.numel() != m:
        _fail(op, f"row scale has {f.RowScale.numel()} elements for {m} rows")
    for t in (f.Mul, f.Residual):
        if t is not None and not (t.dim() == 2 and t.shape[0] == m and t.shape[1] == n):
            _fail(op, f"Mul/Residual must be [{m}×{n}], got {list(t.shape)}")
    out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    if out.numel() == 0:
        return out
    if x.stride(1) != 1:
        x = x.contiguous()
    if w.stride(1) == 1:
        transposed, ldw, wt = 0, w.stride(0), w
    elif w.stride(0) == 1:
        transposed, ldw, wt = 1, w.stride(1), w
    else:
        transposed, wt = 0, w.contiguous()
        ldw = wt.stride(0)
    keep = []

    def cont(t):
        if t is None:
            return None
        t = t.contiguous()
        keep.append(t)
        return t

    bias, rs, mul, res = cont(f.Bias), cont(f.RowScale), cont(f.Mul), cont(f.Residual)
    epi = _lib.Epilogue(_ptr(bias), _ptr(rs), int(f.Act), _ptr(mul), n, _ptr(res), n)
    _lib.check(_lib.lib().fg_matmul(m, n, k, x.data_ptr(), x.stride(0), wt.data_ptr(), ldw,
                                    transposed, out.data_ptr(), n, C.byref(epi), precision,
                                    _stream(x)))
    return out


def MatMul(x: torch.Tensor, w: torch.Tensor, precision: int = PREC_SPLIT) -> torch.Tensor:
    """x · w for 2-D operands (tensor/matmul.go:19)."""
    return MatMulFused(x, w, Fused(), precision)


def RowSumSquares(x: torch.Tensor) -> torch.Tensor:
    """Σ x² per row of a 2-D tensor (matmul_fused.go:125-143)."""
    op = "RowSumSquares"
    _f32_cuda(op, "x", x)
    if x.dim() != 2:
        _fail(op, f"expected a 2-D tensor, got {list(x.shape)}")
    if x.stride(1) != 1:
        x = x.contiguous()
    out = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().fg_row_sum_squares(x.data_ptr(), x.shape[0], x.shape[1], x.stride(0),
                                             out.data_ptr(), _stream(x)))
    return out


def RMSNorm(x: torch.Tensor, g: torch.Tensor, eps: float) -> torch.Tensor:
    """x / √(mean(x²) + eps) · g over the last dimension (attention.go:292-337)."""
    op = "RMSNorm"
    _f32_cuda(op, "x", x)
    if x.dim() == 0:
        _fail(op, "expected at least a 1-D input")
    n = x.shape[-1]
    if g.numel() != n:
        _fail(op, f"g must have {n} elements, got {g.numel()}")
    xc = x.contiguous()
    gc = g.contiguous()
    out = torch.empty_like(xc)
    rows = xc.numel() // n if n else 0
    _lib.check(_lib.lib().fg_rmsnorm(xc.data_ptr(), rows, n, gc.data_ptr(), float(eps),
                                     out.data_ptr(), _stream(x)))
    return out


def RoPE(x: torch.Tensor, base: float, positions: Sequence[int]) -> torch.Tensor:
    """Rotate-half rotary embedding of [..., T, D] (tensor/rope.go:20-87)."""
    op = "RoPE"
    _f32_cuda(op, "x", x)
    if x.dim() < 2:
        _fail(op, f"expected at least a 2-D input, got {list(x.shape)}")
    T, D = x.shape[-2], x.shape[-1]
    if D % 2 != 0:
        _fail(op, f"head dimension {D} must be even")
    if len(positions) != T:
        _fail(op, f"got {len(positions)} positions for {T} slots")
    xc = x.contiguous()
    out = torch.empty_like(xc)
    pos = (C.c_int32 * T)(*[int(p) for p in positions])
    rows = xc.numel() // D
    _lib.check(_lib.lib().fg_rope(xc.data_ptr(), rows, T, D, float(base),
                                  C.cast(pos, C.c_void_p), out.data_ptr(), _stream(x)))
    return out


def AttentionScaled(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    key_lengths: Optional[torch.Tensor] = None, window: int = 0,
                    scale: Optional[float] = None,
                    precision: int = PREC_SPLIT) -> torch.Tensor:
    """softmax(scale·q·kᵀ + mask)·v (attention.go:67) for q [B,Hq,T,D] and
    k, v [B,Hkv,S,D] (grouped-query heads share a KV head, the reference's
    Expand view). The mask is PaddingMask(key_lengths) + WindowMask(window).
    """
    op = "Attention"
    for name, t in (("q", q), ("k", k), ("v", v)):
        _f32_cuda(op, name, t)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        _fail(op, f"q, k, v must be 4-D, got {list(q.shape)} {list(k.shape)} {list(v.shape)}")
    B, Hq, T, D = q.shape
    Bk, Hkv, S, Dk = k.shape
    if Bk != B or Dk != D or tuple(v.shape) != (B, Hkv, S, D):
        _fail(op, f"shapes do not match: q {list(q.shape)}, k {list(k.shape)}, v {list(v.shape)}")
    if Hkv == 0 or Hq % Hkv != 0:
        _fail(op, f"{Hq} query heads not a multiple of {Hkv} key/value heads")
    if scale is None:
        scale = 1.0 / float(D) ** 0.5
    out = torch.empty((B, Hq, T, D), dtype=torch.float32, device=q.device)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    lens = None
    if key_lengths is not None:
        lens = key_lengths.to(device=q.device, dtype=torch.int32).contiguous()
        if lens.numel() != B:
            _fail(op, f"{lens.numel()} key lengths for batch {B}")
    _lib.check(_lib.lib().fg_attention(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), B, Hq, Hkv, T,
                                       S, D, _ptr(lens), int(window), float(scale),
                                       out.data_ptr(), precision, _stream(q)))
    return out
