"""Sparse forms of the head's output for indexing (csrc/sparse.cu).

Upstream (hhkbble/sparton training/model.py:141-144) ``encode`` runs the
model under ``no_grad`` and returns the dense ``reps [B, V]``;
training/train.py:205-210 logs ``(reps > 0).float().mean()``. An inverted
index wants each row's nonzero (vocab id, weight) pairs, or its k heaviest:

* ``reps_to_csr(reps, threshold=0.0)`` -> ``torch.sparse_csr_tensor`` of the
  entries ``> threshold`` (with threshold 0, ``reps.to_sparse_csr()`` of the
  head's non-negative output): columns ascending in every row, int64 row
  pointers, int32 vocab ids, values in reps' dtype. Reads nnz back to size the
  output (one host synchronisation, as ``to_sparse_csr`` has).
* ``csr_arrays(reps, threshold=0.0)`` -> ``(crow, cols, vals)``: the same
  three arrays.
* ``topk_reps(reps, k)`` -> ``(values [B, k], indices [B, k] int32)``: every
  row's k largest entries, by value descending and, among equal values, vocab
  id ascending (``torch.topk`` leaves that order unspecified). No host
  synchronisation.
* ``nonzero_ratio(reps)`` -> fp32 scalar tensor, ``(reps > 0).float().mean()``
  from the CSR row counts (train.py:205-210).
* ``encode_sparse(head, hidden_states, attention_mask, k=None)``: the
  ``no_grad`` forward of a ``SpartonHead`` followed by ``topk_reps`` (k given)
  or ``reps_to_csr``.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _check(reps: torch.Tensor) -> torch.Tensor:
    _require(reps.is_cuda, "the sparse forms only support CUDA tensors")
    _require(reps.dim() == 2, f"reps must be [B, V], got {tuple(reps.shape)}")
    _require(reps.dtype in _lib.DTYPE, f"unsupported dtype {reps.dtype}")
    return reps.contiguous()


def csr_arrays(reps: torch.Tensor, threshold: float = 0.0
               ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(crow [B+1] int64, cols [nnz] int32, vals [nnz]) of the entries > threshold."""
    reps = _check(reps)
    lib = _lib.load()
    B, V = reps.shape
    dev = reps.device
    dt = _lib.DTYPE[reps.dtype]
    crow = torch.empty(B + 1, dtype=torch.int64, device=dev)
    ws = _lib.zeroed_workspace(dev, lib.sparton_sparse_workspace_size(B, V), "csr")
    sh = _lib.stream_handle(dev)
    with torch.cuda.device(dev):
        _lib.check(lib.sparton_reps_csr(_lib.ptr(reps), dt, B, V, float(threshold),
                                        _lib.ptr(crow), None, None, 0, _lib.ptr(ws), ws.numel(),
                                        sh), "sparton_reps_csr (count)")
        nnz = int(crow[B].item())
        cols = torch.empty(nnz, dtype=torch.int32, device=dev)
        vals = torch.empty(nnz, dtype=reps.dtype, device=dev)
        if nnz > 0:
            _lib.check(lib.sparton_reps_csr(_lib.ptr(reps), dt, B, V, float(threshold),
                                            _lib.ptr(crow), _lib.ptr(cols), _lib.ptr(vals), nnz,
                                            _lib.ptr(ws), ws.numel(), sh), "sparton_reps_csr")
    return crow, cols, vals


def reps_to_csr(reps: torch.Tensor, threshold: float = 0.0) -> torch.Tensor:
    """``torch.sparse_csr_tensor`` [B, V] of the entries > threshold."""
    crow, cols, vals = csr_arrays(reps, threshold)
    return torch.sparse_csr_tensor(crow, cols, vals, size=tuple(reps.shape))


def topk_reps(reps: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(values [B, k], indices [B, k] int32): the k largest entries of every row."""
    reps = _check(reps)
    B, V = reps.shape
    _require(0 <= k <= V, f"k={k} must lie in [0, V={V}]")
    lib = _lib.load()
    dev = reps.device
    vals = torch.empty(B, k, dtype=reps.dtype, device=dev)
    idx = torch.empty(B, k, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        st = lib.sparton_reps_topk(_lib.ptr(reps), _lib.DTYPE[reps.dtype], B, V, k,
                                   _lib.ptr(vals), _lib.ptr(idx), _lib.stream_handle(dev))
    _lib.check(st, "sparton_reps_topk")
    return vals, idx


def nonzero_ratio(reps: torch.Tensor) -> torch.Tensor:
    """Fraction of entries > 0 (fp32 scalar on reps' device), from the CSR row
    counts alone (no column or value output)."""
    reps = _check(reps)
    lib = _lib.load()
    B, V = reps.shape
    dev = reps.device
    crow = torch.empty(B + 1, dtype=torch.int64, device=dev)
    ws = _lib.zeroed_workspace(dev, lib.sparton_sparse_workspace_size(B, V), "csr")
    with torch.cuda.device(dev):
        st = lib.sparton_reps_csr(_lib.ptr(reps), _lib.DTYPE[reps.dtype], B, V, 0.0,
                                  _lib.ptr(crow), None, None, 0, _lib.ptr(ws), ws.numel(),
                                  _lib.stream_handle(dev))
    _lib.check(st, "sparton_reps_csr (count)")
    return crow[B].to(torch.float32) / max(B * V, 1)


def encode_sparse(head, hidden_states: torch.Tensor, attention_mask: torch.Tensor,
                  k: Optional[int] = None):
    """``no_grad`` forward of ``head`` (a SpartonHead; its vocabulary shard when
    sharded) and the sparse form of its reps: ``topk_reps(reps, k)`` when k is
    given, else ``reps_to_csr(reps)``."""
    with torch.no_grad():
        reps = head(hidden_states, attention_mask)
    return topk_reps(reps, k) if k is not None else reps_to_csr(reps)
