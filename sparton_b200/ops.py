"""Torch operators of the head, bound to the native C ABI.

Mirrors the custom-op boundary of hhkbble/sparton
(src/sparton/sparton_kernel.py:643-707):

* ``torch.ops.sparton.fused_sparton_fwd(hidden, embed, bias, mask)
  -> (scores[B,V], idx[B,V])``                                    (:643-661)
* ``torch.ops.sparton.fused_sparton_bwd(grad_out, max_scores, max_idx, hidden,
  embed, bias, mask) -> (d_hidden, d_embed, d_bias)``             (:663-694)
* autograd registration linking the two                           (:696-707)

Same op names, argument order and meaning. Differences, all deliberate:

* ``bias`` may be ``None`` (upstream's backward calls ``zeros_like(bias)`` at
  :678 and so cannot train a head without bias).
* ``idx`` is int32 (upstream int64); positions are < 2^31.
* The backward returns gradients in the dtype of the corresponding input.
  Upstream returns fp32 tensors and the autograd engine casts them to the
  input dtype, so the gradients a user sees are the same; d_bias is an empty
  tensor when ``bias`` is None.
* Arguments are validated with ``ValueError`` instead of ``assert``.

The implementation functions ``forward_impl`` / ``backward_impl`` are also used
by the vocabulary-sharded head, which needs fp32 partial d_hidden for its
all-reduce.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def kernel_mask(mask: torch.Tensor) -> torch.Tensor:
    """The mask as a contiguous tensor of a dtype the kernels read directly."""
    if mask.dtype not in _lib.MASK_DTYPE:
        mask = mask != 0
    return mask.contiguous()


def _check_fwd_args(hidden, embed, bias, mask) -> None:
    _require(hidden.is_cuda, "sparton::fused_sparton_fwd only supports CUDA tensors")
    _require(hidden.dim() == 3, f"hidden must be [B,S,D], got shape {tuple(hidden.shape)}")
    _require(embed.dim() == 2, f"embed must be [V,D], got shape {tuple(embed.shape)}")
    _require(hidden.shape[2] == embed.shape[1],
             f"hidden size mismatch: hidden D={hidden.shape[2]}, embed D={embed.shape[1]}")
    _require(hidden.dtype in _lib.DTYPE, f"unsupported dtype {hidden.dtype}")
    _require(embed.dtype == hidden.dtype,
             f"embed dtype {embed.dtype} must equal hidden dtype {hidden.dtype}")
    _require(embed.device == hidden.device, "embed must be on the same device as hidden")
    if bias is not None:
        _require(bias.shape == (embed.shape[0],), f"bias must be [V], got {tuple(bias.shape)}")
        _require(bias.dtype == hidden.dtype,
                 f"bias dtype {bias.dtype} must equal hidden dtype {hidden.dtype}")
        _require(bias.device == hidden.device, "bias must be on the same device as hidden")
    _require(mask.shape == hidden.shape[:2],
             f"mask must be [B,S]={tuple(hidden.shape[:2])}, got {tuple(mask.shape)}")
    _require(mask.device == hidden.device, "mask must be on the same device as hidden")


def forward_impl(hidden: torch.Tensor, embed: torch.Tensor, bias: Optional[torch.Tensor],
                 mask: torch.Tensor, with_idx: bool = True, keep_workspace: bool = False):
    """(reps, idx); with ``with_idx=False`` the inference forward: the kernel
    keeps the max alone, stores reps only and idx is None (no [B, V] int32 is
    allocated or written). ``keep_workspace``: also return the forward's
    workspace (its packed-position layout, which the vocabulary-sharded
    backward reads), as a third element."""
    _check_fwd_args(hidden, embed, bias, mask)
    lib = _lib.load()
    B, S, D = hidden.shape
    V = embed.shape[0]
    hidden = hidden.contiguous()
    embed = embed.contiguous()
    bias = bias.contiguous() if bias is not None else None
    mask = kernel_mask(mask)
    dev = hidden.device
    reps = torch.empty((B, V), dtype=hidden.dtype, device=dev)
    idx = torch.empty((B, V), dtype=torch.int32, device=dev) if with_idx else None
    ws = torch.empty(lib.sparton_fwd_workspace_size(B, S, D, V), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        st = lib.sparton_fwd(_lib.ptr(hidden), _lib.ptr(embed), _lib.ptr(bias), _lib.ptr(mask),
                             _lib.MASK_DTYPE[mask.dtype], _lib.DTYPE[hidden.dtype], B, S, D, V,
                             _lib.ptr(reps), _lib.ptr(idx), _lib.ptr(ws), ws.numel(),
                             _lib.stream_handle(dev))
    _lib.check(st, "sparton_fwd")
    return (reps, idx, ws) if keep_workspace else (reps, idx)


def backward_impl(grad_out: torch.Tensor, scores: torch.Tensor, idx: torch.Tensor,
                  hidden: torch.Tensor, embed: torch.Tensor, has_bias: bool,
                  need_hidden: bool = True, need_embed: bool = True,
                  hidden_grad_dtype: Optional[torch.dtype] = None
                  ) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor], Optional[torch.Tensor]]:
    """(d_hidden, d_embed, d_bias); entries not requested are None.

    d_hidden is produced in ``hidden_grad_dtype`` (default: hidden's dtype; fp32
    for the sharded head's all-reduce); d_embed and d_bias in embed's dtype."""
    _require(grad_out.is_cuda, "sparton::fused_sparton_bwd only supports CUDA tensors")
    lib = _lib.load()
    B, S, D = hidden.shape
    V = embed.shape[0]
    _require(scores.shape == (B, V) and idx.shape == (B, V) and grad_out.shape == (B, V),
             "grad_out, max_scores and max_idx must be [B,V]")
    _require(idx.dtype == torch.int32, f"max_idx must be int32, got {idx.dtype}")
    dtype = hidden.dtype
    gdt = hidden_grad_dtype or dtype
    _require(gdt in (dtype, torch.float32), "hidden_grad_dtype must be hidden's dtype or float32")
    dev = hidden.device
    grad_out = grad_out.to(dtype).contiguous()  # upstream: grad_out.contiguous() (:674)
    scores = scores.contiguous()
    idx = idx.contiguous()
    hidden = hidden.contiguous()
    embed = embed.contiguous()
    d_hidden = torch.empty((B, S, D), dtype=gdt, device=dev) if need_hidden else None
    d_embed = torch.empty((V, D), dtype=dtype, device=dev) if need_embed else None
    d_bias = torch.empty((V,), dtype=dtype, device=dev) if has_bias else None
    ws = torch.empty(lib.sparton_bwd_workspace_size(B, S, D, V), dtype=torch.uint8, device=dev)

    def call(dh, de, dbias, stream_handle):
        return lib.sparton_bwd(_lib.ptr(grad_out), _lib.ptr(scores), _lib.ptr(idx),
                               _lib.ptr(hidden), _lib.ptr(embed), _lib.DTYPE[dtype], B, S, D, V,
                               _lib.ptr(dh), _lib.ptr(de), _lib.ptr(dbias), _lib.DTYPE[gdt],
                               _lib.DTYPE[dtype], _lib.ptr(ws), ws.numel(), stream_handle)

    with torch.cuda.device(dev):
        cur = torch.cuda.current_stream(dev)
        if d_hidden is not None and (d_embed is not None or d_bias is not None):
            # The d_hidden half (sort + dH gather) on the current stream and the
            # d_embed / d_bias half (transpose + dW gather) on a side stream:
            # they read the same inputs and write disjoint parts of the
            # workspace, and together they fill the tail of the persistent dH
            # kernel (cfg2: 0.84 vs 0.88 ms). The current stream waits for
            # both before anything later runs on it.
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(cur)
            st = call(d_hidden, None, None, cur.cuda_stream)
            if st == _lib.OK:
                st = call(None, d_embed, d_bias, side.cuda_stream)
            cur.wait_stream(side)
        else:
            st = call(d_hidden, d_embed, d_bias, cur.cuda_stream)
    _lib.check(st, "sparton_bwd")
    return d_hidden, d_embed, d_bias


def hidden_grad_rows(grad_out: torch.Tensor, scores: torch.Tensor, idx: torch.Tensor,
                     hidden: torch.Tensor, embed: torch.Tensor, out: torch.Tensor, b0: int,
                     b1: int, workspace: Optional[torch.Tensor] = None) -> None:
    """Partial d_hidden of the batch rows [b0, b1) written into ``out[b0:b1]``
    (``out``: [B, S, D] in hidden's dtype or fp32). The backward's rows are
    independent, so this is ``sparton_bwd`` on the row slices with only d_hidden
    requested; the vocab-sharded head uses it to all-reduce finished row
    chunks while the next chunk is computed. All tensors contiguous, on one
    device; ``workspace`` (optional) holds at least
    ``sparton_bwd_workspace_size(b1 - b0, S, D, V)`` bytes."""
    lib = _lib.load()
    B, S, D = hidden.shape
    V = embed.shape[0]
    _require(0 <= b0 <= b1 <= B, f"bad batch row range [{b0}, {b1}) of {B}")
    _require(out.shape == (B, S, D) and out.is_contiguous(), "out must be a contiguous [B,S,D]")
    n = b1 - b0
    if n == 0:
        return
    need = lib.sparton_bwd_workspace_size(n, S, D, V)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=hidden.device)
    dev = hidden.device
    with torch.cuda.device(dev):
        st = lib.sparton_bwd(_lib.ptr(grad_out[b0:b1]), _lib.ptr(scores[b0:b1]),
                             _lib.ptr(idx[b0:b1]), _lib.ptr(hidden[b0:b1]), _lib.ptr(embed),
                             _lib.DTYPE[hidden.dtype], n, S, D, V, _lib.ptr(out[b0:b1]), None,
                             None, _lib.DTYPE[out.dtype], _lib.DTYPE[hidden.dtype],
                             _lib.ptr(workspace), workspace.numel(), _lib.stream_handle(dev))
    _lib.check(st, "sparton_bwd (d_hidden rows)")


@torch.library.custom_op("sparton::fused_sparton_fwd", mutates_args=())
def fused_sparton_fwd(hidden: torch.Tensor, embed: torch.Tensor, bias: Optional[torch.Tensor],
                      mask: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """scores[b,v] = max_s log1p(relu((hidden[b,s]·embed[v] + bias[v]) * mask[b,s])),
    idx[b,v] = first s attaining it (0 when the max is <= 0)."""
    return forward_impl(hidden, embed, bias, mask)


@fused_sparton_fwd.register_fake
def _(hidden, embed, bias, mask):
    B, S, D = hidden.shape
    V = embed.shape[0]
    return hidden.new_empty((B, V)), torch.empty((B, V), device=hidden.device, dtype=torch.int32)


@torch.library.custom_op("sparton::fused_sparton_bwd", mutates_args=())
def fused_sparton_bwd(grad_out: torch.Tensor, max_scores: torch.Tensor, max_idx: torch.Tensor,
                      hidden: torch.Tensor, embed: torch.Tensor, bias: Optional[torch.Tensor],
                      mask: torch.Tensor, need_hidden: bool = True, need_embed: bool = True,
                      need_bias: bool = True) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients of fused_sparton_fwd w.r.t. hidden, embed and bias. ``mask`` is
    accepted for signature symmetry with upstream (:671) and not read: positions
    with mask 0 never hold the argmax. The ``need_*`` flags (not in upstream;
    default True) skip a gradient, which is then returned as an empty tensor,
    as d_bias is when ``bias`` is None."""
    d_hidden, d_embed, d_bias = backward_impl(grad_out, max_scores, max_idx, hidden, embed,
                                              bias is not None and need_bias,
                                              need_hidden=need_hidden, need_embed=need_embed)
    empty = hidden.new_empty((0,))
    return (d_hidden if d_hidden is not None else empty,
            d_embed if d_embed is not None else empty,
            d_bias if d_bias is not None else empty)


@fused_sparton_bwd.register_fake
def _(grad_out, max_scores, max_idx, hidden, embed, bias, mask, need_hidden=True,
      need_embed=True, need_bias=True):
    empty = hidden.new_empty((0,))
    return (torch.empty_like(hidden) if need_hidden else empty,
            torch.empty_like(embed) if need_embed else empty,
            torch.empty_like(bias) if (bias is not None and need_bias) else empty)


def _setup_context(ctx, inputs, output):
    hidden, embed, bias, mask = inputs
    scores, idx = output
    ctx.has_bias = bias is not None
    ctx.save_for_backward(scores, idx, hidden, embed, bias, mask)


def _backward(ctx, grad_scores, grad_idx):
    # grad_idx is ignored: idx is not differentiable (upstream :701-705).
    scores, idx, hidden, embed, bias, mask = ctx.saved_tensors
    need_h, need_e = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
    need_b = ctx.has_bias and ctx.needs_input_grad[2]
    if not (need_h or need_e or need_b):
        return None, None, None, None
    d_hidden, d_embed, d_bias = fused_sparton_bwd(grad_scores, scores, idx, hidden, embed,
                                                  bias, mask, need_hidden=need_h,
                                                  need_embed=need_e, need_bias=need_b)
    return (d_hidden if need_h else None, d_embed if need_e else None,
            d_bias if need_b else None, None)


fused_sparton_fwd.register_autograd(_backward, setup_context=_setup_context)


@torch.library.custom_op("sparton::fused_sparton_fwd_scores", mutates_args=())
def fused_sparton_fwd_scores(hidden: torch.Tensor, embed: torch.Tensor,
                             bias: Optional[torch.Tensor], mask: torch.Tensor) -> torch.Tensor:
    """Inference forward: scores[B,V] of fused_sparton_fwd without the argmax.
    Upstream's counterpart is its no-argmax ``fused_sparton_fwd`` host function
    (sparton_kernel.py:372-394, reduce kernel :257-334), meant for ``encode``
    under ``no_grad`` (training/model.py:141-144). Not differentiable: training
    uses ``fused_sparton_fwd``, whose idx the backward needs."""
    return forward_impl(hidden, embed, bias, mask, with_idx=False)[0]


@fused_sparton_fwd_scores.register_fake
def _(hidden, embed, bias, mask):
    return hidden.new_empty((hidden.shape[0], embed.shape[0]))
