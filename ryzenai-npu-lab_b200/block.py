"""Torch-facing wrappers of the layer kernels around the attention path
(include/b2_block.h): projection GEMM (optionally with the SwiGLU gate),
residual add + RMSNorm, SwiGLU gate, short-convolution decode step, greedy
argmax over the logits.  Same conventions as attention.py: host checks raise ValueError,
library refusals raise B2Error, work is queued on the current CUDA stream."""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .attention import _need, _ptr, _stream


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor | None, gamma: torch.Tensor, eps: float, *,
                out: torch.Tensor, sum_out: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """out = gamma * bf16(s * rsqrt(mean(s^2) + eps)) with s = bf16(x + residual)
    (s = x without a residual); s is also written to sum_out (which may be
    the residual or x itself).  x, residual, out, sum_out: bf16 [rows, width]."""
    dev = x.device
    if x.dim() != 2:
        raise ValueError("x must be [rows, width]")
    rows, width = x.shape
    _need(x, "x", torch.bfloat16, dev)
    if residual is not None:
        _need(residual, "residual", torch.bfloat16, dev, (rows, width))
    if sum_out is not None:
        _need(sum_out, "sum_out", torch.bfloat16, dev, (rows, width))
    _need(gamma, "gamma", torch.bfloat16, dev, (width,))
    _need(out, "out", torch.bfloat16, dev, (rows, width))
    rc = _lib.load().b2_add_rmsnorm(_ptr(x), _ptr(residual), _ptr(gamma), ctypes.c_float(eps), _ptr(sum_out),
                                    _ptr(out), rows, width, _stream(dev, stream))
    _lib.check(rc, "b2_add_rmsnorm")
    return out


def _rows(t: torch.Tensor, name: str, device: torch.device) -> int:
    """Row stride of a bf16 matrix whose rows are contiguous (a row-sliced view is fine)."""
    if not isinstance(t, torch.Tensor) or t.dim() != 2:
        raise ValueError(f"{name} must be a 2-D tensor")
    if t.dtype != torch.bfloat16 or t.device != device:
        raise ValueError(f"{name} must be bf16 on {device}")
    if t.stride(1) != 1 and t.shape[1] > 1:
        raise ValueError(f"{name} must have contiguous rows")
    return t.stride(0) if t.shape[0] > 1 else t.shape[1]


def gemm_plan(m: int, n: int, k: int, mode: int = _lib.B2_GEMM_PLAIN, tile_n: int = 0,
              splits: int = 0) -> tuple[int, int, int]:
    """(tile_n, splits, ctas) that b2_gemm uses for an m x n x k product."""
    t, s, c = ctypes.c_int32(tile_n), ctypes.c_int32(splits), ctypes.c_int32(0)
    _lib.check(_lib.load().b2_gemm_plan(m, n, k, mode, ctypes.byref(t), ctypes.byref(s), ctypes.byref(c)),
               "b2_gemm_plan")
    return t.value, s.value, c.value


def gemm(a: torch.Tensor, w: torch.Tensor, *, out: torch.Tensor, dev_err: torch.Tensor, swiglu: bool = False,
         tile_n: int = 0, splits: int = 0, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """out = a @ w.T on the tensor cores (bf16 [m, k] x bf16 [n, k] -> bf16
    [m, n], fp32 accumulation).  swiglu: w = [w1; w3] ([2 n, k]) and out =
    bf16(bf16(silu(a w1^T)) * bf16(a w3^T)).  Rows may be strided (row-sliced
    views); k % 64 == 0.  dev_err: int32 [1] (B2_DEV_TIMEOUT if a wait gives up)."""
    dev = a.device
    lda, ldw, ldd = _rows(a, "a", dev), _rows(w, "w", dev), _rows(out, "out", dev)
    m, k = a.shape
    n = w.shape[0] // 2 if swiglu else w.shape[0]
    if w.shape[1] != k or (swiglu and w.shape[0] % 2):
        raise ValueError(f"w must be [{'2 n' if swiglu else 'n'}, {k}], got {tuple(w.shape)}")
    if tuple(out.shape) != (m, n):
        raise ValueError(f"out must be [{m}, {n}], got {tuple(out.shape)}")
    _need(dev_err, "dev_err", torch.int32, dev, (1,))
    mode = _lib.B2_GEMM_SWIGLU if swiglu else _lib.B2_GEMM_PLAIN
    rc = _lib.load().b2_gemm(_ptr(a), lda, _ptr(w), ldw, _ptr(out), ldd, m, n, k, mode, tile_n, splits,
                             _ptr(dev_err), _stream(dev, stream))
    _lib.check(rc, "b2_gemm")
    return out


def swiglu(gu: torch.Tensor, *, out: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """out = bf16(bf16(silu(g)) * u) for gu = [g | u] (bf16 [rows, 2 * ffn]) -> bf16 [rows, ffn]."""
    dev = gu.device
    if gu.dim() != 2 or gu.shape[1] % 2:
        raise ValueError("gu must be [rows, 2 * ffn]")
    rows, ffn = gu.shape[0], gu.shape[1] // 2
    _need(gu, "gu", torch.bfloat16, dev)
    _need(out, "out", torch.bfloat16, dev, (rows, ffn))
    _lib.check(_lib.load().b2_swiglu(_ptr(gu), _ptr(out), rows, ffn, _stream(dev, stream)), "b2_swiglu")
    return out


def shortconv_step(bcx: torch.Tensor, conv_state: torch.Tensor, conv_w: torch.Tensor, *, out: torch.Tensor,
                   stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """One decode step of the gated short convolution: bcx = [B | C | x]
    (bf16 [rows, 3 * hidden]), conv_state bf16 [rows, hidden, 3] (rolled in
    place), conv_w bf16 [hidden, 3] -> out bf16 [rows, hidden]."""
    dev = bcx.device
    if bcx.dim() != 2 or bcx.shape[1] % 3:
        raise ValueError("bcx must be [rows, 3 * hidden]")
    rows, hidden = bcx.shape[0], bcx.shape[1] // 3
    _need(bcx, "bcx", torch.bfloat16, dev)
    _need(conv_state, "conv_state", torch.bfloat16, dev, (rows, hidden, 3))
    _need(conv_w, "conv_w", torch.bfloat16, dev, (hidden, 3))
    _need(out, "out", torch.bfloat16, dev, (rows, hidden))
    rc = _lib.load().b2_shortconv_step(_ptr(bcx), _ptr(conv_state), _ptr(conv_w), _ptr(out), rows, hidden,
                                       _stream(dev, stream))
    _lib.check(rc, "b2_shortconv_step")
    return out


def argmax_rows(logits: torch.Tensor, *, out: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """out[r] = torch.argmax(logits[r]) for bf16 logits [rows, cols] -> int64 [rows]."""
    dev = logits.device
    if logits.dim() != 2:
        raise ValueError("logits must be [rows, cols]")
    rows, cols = logits.shape
    _need(logits, "logits", torch.bfloat16, dev)
    _need(out, "out", torch.int64, dev, (rows,))
    _lib.check(_lib.load().b2_argmax_rows(_ptr(logits), rows, cols, _ptr(out), _stream(dev, stream)),
               "b2_argmax_rows")
    return out
