"""Tensor-core GEMM for the contractions around the head (``sparton_gemm`` of
the C ABI): the MLM transform's dense layer and its backward products, and the
InfoNCE scores and their backward. Upstream computes these with torch matmuls
(training/model.py:25-35 and :82-85; training/train.py:73-77).

``gemm(A, B)`` computes ``A @ B.T`` for 16-bit ``A`` [M, K] and ``B`` [N, K]
with fp32 sums; either operand may instead be passed through its transpose's
storage (``a_t`` / ``b_t``: the tensor given is [K, M] / [K, N], contiguous),
which is how the backward products read their inputs without copies.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib


def _rows(t: torch.Tensor) -> torch.Tensor:
    """``t`` with contiguous rows (a strided view of a padded buffer is kept)."""
    return t if t.dim() == 2 and t.stride(1) == 1 and t.stride(0) >= t.shape[1] else t.contiguous()


def gemm(a: torch.Tensor, b: torch.Tensor, *, a_t: bool = False, b_t: bool = False,
         bias: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
         out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """C[M, N] = A @ B.T (+ bias).

    a: [M, K], or with ``a_t`` the [K, M] tensor holding A.T; b: [N, K], or with
    ``b_t`` the [K, N] tensor holding B.T. Each may be a row-contiguous view of
    a wider buffer (its rows then hold ``stride(0)`` elements, which must be a
    multiple of 8; a view narrower than its rows in the contraction dimension
    needs zeros in the padding). bias: [N] (operand dtype) or None. The result is
    ``out_dtype`` (default: the operand dtype; float32 allowed), or written into
    ``out`` ([M, N], rows contiguous)."""
    if a.dtype not in (torch.bfloat16, torch.float16) or b.dtype != a.dtype:
        raise ValueError(f"gemm takes bf16 / f16 operands of one dtype, got {a.dtype}, {b.dtype}")
    if not (a.is_cuda and b.is_cuda):
        raise ValueError("gemm only supports CUDA tensors")
    a = _rows(a)
    b = _rows(b)
    M, K = (a.shape[1], a.shape[0]) if a_t else (a.shape[0], a.shape[1])
    N, Kb = (b.shape[1], b.shape[0]) if b_t else (b.shape[0], b.shape[1])
    if K != Kb:
        raise ValueError(f"contraction sizes differ: {K} vs {Kb}")
    if bias is not None:
        bias = bias.to(a.dtype).contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype or a.dtype, device=a.device)
    if out.shape != (M, N) or out.stride(1) != 1:
        raise ValueError("out must be [M, N] with contiguous rows")
    lib = _lib.load()
    dev = a.device
    ws = torch.empty(max(lib.sparton_gemm_workspace_size(M, N, K), 256), dtype=torch.uint8,
                     device=dev)
    with torch.cuda.device(dev):
        st = lib.sparton_gemm(_lib.ptr(a), _lib.LAYOUT_COLS if a_t else _lib.LAYOUT_ROWS,
                              a.stride(0), _lib.ptr(b),
                              _lib.LAYOUT_COLS if b_t else _lib.LAYOUT_ROWS, b.stride(0),
                              _lib.ptr(bias), _lib.DTYPE[a.dtype], M, N, K, _lib.ptr(out),
                              _lib.DTYPE[out.dtype], out.stride(0), _lib.ptr(ws), ws.numel(),
                              _lib.stream_handle(dev))
    _lib.check(st, "sparton_gemm")
    return out


def padded(t: torch.Tensor, mult: int = 64) -> torch.Tensor:
    """A row-contiguous view [r, c] of ``t`` whose rows hold round_up(c, mult)
    elements, the padding zero (one copy, sparton_pad_rows)."""
    r, c = t.shape
    cp = round_up(c, mult)
    t = t.contiguous()
    if cp == c:
        return t
    buf = torch.empty((r, cp), dtype=t.dtype, device=t.device)
    if t.dtype in (torch.bfloat16, torch.float16) and t.is_cuda:
        with torch.cuda.device(t.device):
            _lib.check(_lib.load().sparton_pad_rows(_lib.ptr(t), _lib.DTYPE[t.dtype], r, c,
                                                    _lib.ptr(buf), cp,
                                                    _lib.stream_handle(t.device)),
                       "sparton_pad_rows")
    else:
        buf[:, c:].zero_()
        buf[:, :c].copy_(t)
    return buf[:, :c]


def round_up(x: int, m: int) -> int:
    return -(-x // m) * m
