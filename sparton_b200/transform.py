"""The MLM transform in front of the head, and the projection module that
chains it to ``SpartonHead`` — hhkbble/sparton training/model.py:7-45 (the
transform of BERT's ``cls.predictions`` and RoBERTa's ``lm_head``: dense →
exact-erf gelu → LayerNorm) and ``ProjectionSparton`` (:65-85).

* ``MLMTransform(dense, layer_norm)``: ``h = LayerNorm(gelu(dense(x)))`` with
  the dense layer on the library's tcgen05 GEMM (``sparton_gemm``, bias in its
  epilogue; fp32 inputs stay on ``F.linear``) and gelu + LayerNorm in one
  kernel (``sparton_transform_fwd``, csrc/transform.cu) that writes the head's
  input and saves each row's mean / rstd; the backward is one kernel (d of
  LayerNorm and gelu, and per-CTA column sums) plus a fixed-order reduction
  for d_gamma / d_beta / d_dense_bias (``sparton_transform_bwd``) and two
  tcgen05 GEMMs for d_x and d_dense_weight. Parameters are shared with the modules it
  is built from. ``MLMTransform.from_module(transform)`` accepts BERT's
  ``BertPredictionHeadTransform`` (``dense``, ``transform_act_fn``,
  ``LayerNorm``) and the reference's ``RobertaTransform`` (``dense``,
  ``layer_norm``, gelu).
* ``SpartonProjection(transform, decoder)``: drop-in for ``ProjectionSparton``
  (same constructor arguments, same forward), with the transform above and a
  ``SpartonHead`` tied to ``decoder``; keyword-only ``process_group`` /
  ``gather_output`` shard the head's vocabulary.

As in the reference's separate modules, the gelu output is rounded to the
input dtype before the normalisation.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib
from .gemm import gemm
from .head import SpartonHead


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def transform_fwd_impl(y: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float):
    """(h, mean, rstd): gelu + LayerNorm of y [..., D] (sparton_transform_fwd)."""
    _require(y.is_cuda, "the transform only supports CUDA tensors")
    _require(y.dtype in _lib.DTYPE, f"unsupported dtype {y.dtype}")
    lib = _lib.load()
    D = y.shape[-1]
    y = y.contiguous()
    rows = y.numel() // max(D, 1)
    gamma = gamma.to(y.dtype).contiguous()
    beta = beta.to(y.dtype).contiguous()
    dev = y.device
    h = torch.empty_like(y)
    mean = torch.empty(rows, dtype=torch.float32, device=dev)
    rstd = torch.empty(rows, dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        st = lib.sparton_transform_fwd(_lib.ptr(y), _lib.ptr(gamma), _lib.ptr(beta), float(eps),
                                       _lib.DTYPE[y.dtype], rows, D, _lib.ptr(h), _lib.ptr(mean),
                                       _lib.ptr(rstd), _lib.stream_handle(dev))
    _lib.check(st, "sparton_transform_fwd")
    return h, mean, rstd


def transform_bwd_impl(dh: torch.Tensor, y: torch.Tensor, gamma: torch.Tensor,
                       mean: torch.Tensor, rstd: torch.Tensor, need_params: bool = True):
    """(dy, d_gamma, d_beta, d_dense_bias) from dh (sparton_transform_bwd); the
    last three are None without need_params."""
    lib = _lib.load()
    D = y.shape[-1]
    rows = y.numel() // max(D, 1)
    dh = dh.to(y.dtype).contiguous()
    gamma = gamma.to(y.dtype).contiguous()
    dev = y.device
    dy = torch.empty_like(y)
    dg = db = dbias = None
    ws = None
    if need_params:
        dg = torch.empty(D, dtype=y.dtype, device=dev)
        db = torch.empty(D, dtype=y.dtype, device=dev)
        dbias = torch.empty(D, dtype=y.dtype, device=dev)
        ws = torch.empty(max(lib.sparton_transform_workspace_size(rows, D), 1), dtype=torch.uint8,
                         device=dev)
    with torch.cuda.device(dev):
        st = lib.sparton_transform_bwd(_lib.ptr(dh), _lib.ptr(y), _lib.ptr(gamma), _lib.ptr(mean),
                                       _lib.ptr(rstd), _lib.DTYPE[y.dtype], rows, D, _lib.ptr(dy),
                                       _lib.ptr(dg), _lib.ptr(db), _lib.ptr(dbias), _lib.ptr(ws),
                                       0 if ws is None else ws.numel(), _lib.stream_handle(dev))
    _lib.check(st, "sparton_transform_bwd")
    return dy, dg, db, dbias


def _tensor_core(x: torch.Tensor, w: torch.Tensor) -> bool:
    """16-bit operands with 16-byte rows: the dense layer and its backward
    products run on the library's tcgen05 GEMM. fp32 keeps torch's fp32 GEMM
    (tcgen05 has no fp32-exact kind; the fp32 path is held to rtol 1e-5)."""
    return (x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and w.dtype == x.dtype
            and w.shape[0] % 8 == 0 and w.shape[1] % 8 == 0)


def _dense_fwd(x, w, b):
    """y = x @ w.T + b (nn.Linear), on the tensor-core GEMM when it applies."""
    if not _tensor_core(x, w):
        return F.linear(x, w, b)
    lead = x.shape[:-1]
    y = gemm(x.reshape(-1, x.shape[-1]), w, bias=b)
    return y.reshape(*lead, w.shape[0])


def _dense_bwd(dy, x, w, need_x: bool, need_w: bool):
    """(dx = dy @ w, dw = dy.T @ x) of the dense layer; the GEMM reads dy, x
    and w in place (w and, for dw, dy and x through their transposed layout)."""
    D_in = x.shape[-1]
    dy2 = dy.reshape(-1, dy.shape[-1])
    x2 = x.reshape(-1, D_in)
    if not _tensor_core(x, w):
        dx = (dy @ w) if need_x else None
        dw = (dy2.t() @ x2) if need_w else None
        return dx, dw
    dx = gemm(dy2, w, b_t=True).reshape(x.shape) if need_x else None
    dw = gemm(dy2, x2, a_t=True, b_t=True, out_dtype=w.dtype) if need_w else None
    return dx, dw


class _Transform(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dense_w, dense_b, gamma, beta, eps):
        y = _dense_fwd(x, dense_w, dense_b)
        h, mean, rstd = transform_fwd_impl(y, gamma, beta, eps)
        ctx.save_for_backward(x, dense_w, y, gamma, mean, rstd)
        ctx.has_dense_bias = dense_b is not None
        return h

    @staticmethod
    def backward(ctx, dh):
        x, dense_w, y, gamma, mean, rstd = ctx.saved_tensors
        need = ctx.needs_input_grad
        dy, dg, db, dbias = transform_bwd_impl(dh, y, gamma, mean, rstd,
                                               need_params=any(need[2:5]))
        dx, dw = _dense_bwd(dy, x, dense_w, need[0], need[1])
        return (dx, dw, dbias if (need[2] and ctx.has_dense_bias) else None,
                dg if need[3] else None, db if need[4] else None, None)


def _is_exact_gelu(act) -> bool:
    if isinstance(act, nn.GELU):
        return act.approximate == "none"
    name = type(act).__name__
    if name == "GELUActivation":  # transformers' "gelu": exact erf form
        return True
    return getattr(act, "__name__", "") == "gelu" and getattr(act, "__module__", "").startswith(
        "transformers")


class MLMTransform(nn.Module):
    """``h = LayerNorm(gelu(dense(x)))`` on the native kernels; shares the
    parameters of ``dense`` (nn.Linear) and ``layer_norm`` (nn.LayerNorm)."""

    def __init__(self, dense: nn.Linear, layer_norm: nn.LayerNorm):
        super().__init__()
        _require(isinstance(dense, nn.Linear), "dense must be an nn.Linear")
        _require(isinstance(layer_norm, nn.LayerNorm) and layer_norm.elementwise_affine
                 and len(layer_norm.normalized_shape) == 1
                 and layer_norm.normalized_shape[0] == dense.out_features,
                 "layer_norm must be an affine nn.LayerNorm over dense's output")
        self.dense = dense
        self.layer_norm = layer_norm

    @classmethod
    def from_module(cls, transform: nn.Module) -> "MLMTransform":
        """From BERT's predictions.transform or the reference's RobertaTransform."""
        if hasattr(transform, "transform_act_fn") and hasattr(transform, "LayerNorm"):
            _require(_is_exact_gelu(transform.transform_act_fn),
                     f"unsupported activation {type(transform.transform_act_fn).__name__}; "
                     "the transform kernel implements the exact (erf) gelu")
            return cls(transform.dense, transform.LayerNorm)
        if hasattr(transform, "dense") and hasattr(transform, "layer_norm"):
            return cls(transform.dense, transform.layer_norm)  # model.py:25-35: gelu
        raise ValueError(f"unsupported transform module {type(transform).__name__}")

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _Transform.apply(x, self.dense.weight, self.dense.bias, self.layer_norm.weight,
                                self.layer_norm.bias, float(self.layer_norm.eps))


class SpartonProjection(nn.Module):
    """Drop-in for the reference's ``ProjectionSparton(transform, decoder)``
    (training/model.py:65-85): MLM transform + SpartonHead tied to ``decoder``."""

    def __init__(self, transform: nn.Module, decoder: nn.Linear, *,
                 process_group=None, gather_output: bool = False,
                 grad_reduce_dtype: Optional[torch.dtype] = None):
        super().__init__()
        self.transform = MLMTransform.from_module(transform)
        vocab_size, hidden_dim = decoder.out_features, decoder.in_features
        self.sparton_head = SpartonHead(vocab_size, hidden_dim, use_bias=decoder.bias is not None,
                                        process_group=process_group, gather_output=gather_output,
                                        grad_reduce_dtype=grad_reduce_dtype).to(
                                            device=decoder.weight.device)
        self.sparton_head.tie_weights(decoder)

    def forward(self, hidden_states: torch.Tensor, attention_mask: torch.Tensor) -> torch.Tensor:
        return self.sparton_head(self.transform(hidden_states), attention_mask)
