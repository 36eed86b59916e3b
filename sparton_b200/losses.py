"""Training losses that consume the head's output: hhkbble/sparton
training/train.py:73-87, same names and arguments, plus a vocabulary-sharded
form for representations that hold one vocabulary shard per rank (the output
of ``SpartonHead(..., process_group=...)``):

* ``info_nce_loss(query_reps, doc_reps, temperature=1.0, *, process_group=None)``
  (train.py:73-77): ``scores = q @ d.T / temperature``, cross entropy against
  the diagonal (in-batch negatives). Sharded, each rank scores its own
  vocabulary shard and only the small ``[Bq, Bd]`` partial scores are
  all-reduced (sum); the representations are never gathered. The backward is
  local. Scores are accumulated in fp32 (upstream: in the reps' dtype).
* ``l1_regularization(reps, *, process_group=None)`` (:80-82):
  ``mean_b sum_v |reps|``.
* ``flops_regularization(reps, *, process_group=None, vocab_size=None)``
  (:85-87): ``mean_v (sum_b reps)^2``; ``vocab_size`` is the whole
  vocabulary (when omitted with a process group, the shard widths are summed,
  which reads one number back to the host).
* ``regularizers(reps, ...) -> (l1, flops)``: both from one pass over reps
  (``sparton_reg_fwd`` / ``sparton_reg_bwd``, csrc/reg.cu); the two functions
  above call it. Sharded, the two totals are all-reduced.

Loss values are fp32 scalars (upstream: the reps' dtype).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _lib
from .gemm import gemm, padded


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def reg_forward_impl(reps: torch.Tensor, scale_l1: float,
                     scale_flops: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """(colsum [V] fp32, out [2] fp32 = {scale_l1 * sum |reps|,
    scale_flops * sum_v colsum^2})."""
    _require(reps.is_cuda, "the regularisers only support CUDA tensors")
    _require(reps.dim() == 2, f"reps must be [B, V], got {tuple(reps.shape)}")
    _require(reps.dtype in _lib.DTYPE, f"unsupported dtype {reps.dtype}")
    lib = _lib.load()
    reps = reps.contiguous()
    B, V = reps.shape
    dev = reps.device
    colsum = torch.empty(V, dtype=torch.float32, device=dev)
    out = torch.empty(2, dtype=torch.float32, device=dev)
    ws = _lib.zeroed_workspace(dev, lib.sparton_reg_workspace_size(B, V), "reg")
    with torch.cuda.device(dev):
        st = lib.sparton_reg_fwd(_lib.ptr(reps), _lib.DTYPE[reps.dtype], B, V, scale_l1,
                                 scale_flops, _lib.ptr(colsum), _lib.ptr(out), _lib.ptr(ws),
                                 ws.numel(), _lib.stream_handle(dev))
    _lib.check(st, "sparton_reg_fwd")
    return colsum, out


def reg_backward_impl(reps: torch.Tensor, colsum: torch.Tensor, g: torch.Tensor,
                      scale_l1: float, scale_flops: float) -> torch.Tensor:
    """grad = g[0] * scale_l1 * sign(reps) + g[1] * scale_flops * colsum[None, :],
    in reps' dtype (g: the upstream gradients of (l1, flops), fp32 on the device)."""
    lib = _lib.load()
    reps = reps.contiguous()
    B, V = reps.shape
    dev = reps.device
    grad = torch.empty_like(reps)
    g = g.to(device=dev, dtype=torch.float32).contiguous()
    with torch.cuda.device(dev):
        st = lib.sparton_reg_bwd(_lib.ptr(reps), _lib.ptr(colsum), _lib.ptr(g), _lib.ptr(g) + 4,
                                 scale_l1, scale_flops, _lib.DTYPE[reps.dtype], B, V,
                                 _lib.ptr(grad), _lib.stream_handle(dev))
    _lib.check(st, "sparton_reg_bwd")
    return grad


def _vocab_total(width: int, device, group) -> int:
    t = torch.tensor([width], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return int(t.item())


class _Regularizers(torch.autograd.Function):
    @staticmethod
    def forward(ctx, reps, group, vocab_size):
        B, V = reps.shape
        if group is not None:
            V = vocab_size if vocab_size is not None else _vocab_total(V, reps.device, group)
        elif vocab_size is not None:
            V = vocab_size
        # The kernel scales its sums (1/B, 1/V), so a shard's two values add up
        # over the group to the losses.
        colsum, out = reg_forward_impl(reps, 1.0 / B, 1.0 / V)
        if group is not None:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=group)
        ctx.save_for_backward(reps, colsum)
        ctx.B, ctx.V = B, V
        return out

    @staticmethod
    def backward(ctx, g):
        reps, colsum = ctx.saved_tensors
        return reg_backward_impl(reps, colsum, g, 1.0 / ctx.B, 2.0 / ctx.V), None, None


def regularizers(reps: torch.Tensor, *, process_group=None,
                 vocab_size: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(l1, flops) of ``reps`` [B, V] (a vocabulary shard with a process group)."""
    l1, flops = _Regularizers.apply(reps, process_group, vocab_size).unbind(0)
    return l1, flops


def l1_regularization(reps: torch.Tensor, *, process_group=None) -> torch.Tensor:
    """mean_b sum_v |reps[b, v]| (train.py:80-82)."""
    return regularizers(reps, process_group=process_group)[0]


def flops_regularization(reps: torch.Tensor, *, process_group=None,
                         vocab_size: Optional[int] = None) -> torch.Tensor:
    """mean_v (sum_b reps[b, v])^2 (train.py:85-87)."""
    return regularizers(reps, process_group=process_group, vocab_size=vocab_size)[1]


class _Scores(torch.autograd.Function):
    """q @ d.T in fp32, summed over the vocabulary shards of a process group.

    16-bit reps on a GPU run on the library's tcgen05 GEMM: the forward as one
    split-K contraction over the vocabulary with fp32 output, the backward as
    gq = gs @ d and gd = gs.T @ q with gs rounded to the reps' dtype (what the
    reference's bf16 matmul autograd computes, train.py:73-77), both reading d
    and q in place through their transposed layout. The GEMM needs 16-byte
    rows, so q and d are zero-padded once to a vocabulary multiple of 64 and
    batch multiples of 8 (the padding adds zeros to every sum) and kept for the
    backward."""

    @staticmethod
    def forward(ctx, q, d, group):
        Bq, V = q.shape
        Bd = d.shape[0]
        ctx.shapes = (Bq, Bd, V)
        ctx.tc = q.is_cuda and q.dtype in (torch.bfloat16, torch.float16) and d.dtype == q.dtype
        if ctx.tc:
            qv, dv = padded(q), padded(d)  # rows of round_up(V, 64), zero padding
            s = gemm(qv, dv, out_dtype=torch.float32)
            ctx.save_for_backward(qv, dv)
        else:
            s = torch.matmul(q.float(), d.float().t())
            ctx.save_for_backward(q, d)
        if group is not None:
            dist.all_reduce(s, op=dist.ReduceOp.SUM, group=group)
        return s

    @staticmethod
    def backward(ctx, gs):
        Bq, Bd, V = ctx.shapes
        need_q, need_d = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if not ctx.tc:
            q, d = ctx.saved_tensors
            gq = (gs @ d.float()).to(q.dtype) if need_q else None
            gd = (gs.t() @ q.float()).to(d.dtype) if need_d else None
            return gq, gd, None
        qv, dv = ctx.saved_tensors
        gsv = padded(gs.to(qv.dtype), 8)                     # [Bq, Bd], rows of round_up(Bd, 8)
        gq = gemm(gsv, dv, b_t=True) if need_q else None           # gs @ d   -> [Bq, V]
        gd = gemm(gsv, qv, a_t=True, b_t=True) if need_d else None  # gs.T @ q -> [Bd, V]
        return gq, gd, None


def scores(query_reps: torch.Tensor, doc_reps: torch.Tensor, *, process_group=None) -> torch.Tensor:
    """[Bq, Bd] dot products of query and document representations (fp32)."""
    _require(query_reps.dim() == 2 and doc_reps.dim() == 2
             and query_reps.shape[1] == doc_reps.shape[1],
             "query_reps and doc_reps must be [Bq, V] and [Bd, V]")
    return _Scores.apply(query_reps, doc_reps, process_group)


def info_nce_loss(query_reps: torch.Tensor, doc_reps: torch.Tensor, temperature: float = 1.0,
                  *, process_group=None) -> torch.Tensor:
    """In-batch negatives contrastive loss (train.py:73-77). Query i's positive
    is document i, so there must be at least as many documents as queries
    (checked here; upstream's cross_entropy would fail on the device)."""
    _require(query_reps.dim() == 2 and doc_reps.dim() == 2
             and query_reps.shape[0] <= doc_reps.shape[0],
             f"info_nce_loss needs at least as many documents as queries, got "
             f"{tuple(query_reps.shape)} and {tuple(doc_reps.shape)}")
    s = scores(query_reps, doc_reps, process_group=process_group) / temperature
    labels = torch.arange(s.size(0), device=s.device)
    return F.cross_entropy(s, labels)
