"""CPU oracle for the sparse forms of reps — TEST INFRASTRUCTURE ONLY.

Only ``tests/`` and ``bench.py``'s CPU legs may import this module, and only as
the checker; the product path (``sparton_b200.sparse``) never calls it.

The reference returns dense reps (hhkbble/sparton training/model.py:141-144,
``encode``) and measures sparsity as ``(reps > 0).float().mean()``
(training/train.py:205-210); the sparse forms are defined by torch, the
reference's own dependency (pyproject.toml: torch>=2.7.1):

* ``csr``: ``torch.Tensor.to_sparse_csr`` of ``where(reps > threshold, reps,
  0)``: row pointers, column indices ascending inside each row, values;
* ``topk``: the values of ``torch.topk(reps, k, dim=1)`` (sorted, largest
  first), with the order among equal values fixed to vocab id ascending
  (torch leaves it unspecified); NaN above +inf.

Restated in numpy and pinned against fixtures made by torch itself
(tests/golden/make_golden_sparse.py).
"""
from __future__ import annotations

import numpy as np


def csr(reps, threshold: float = 0.0):
    """(crow [B+1] int64, cols [nnz] int64, vals [nnz]) of the entries > threshold."""
    x = np.asarray(reps)
    keep = x > threshold
    crow = np.zeros(x.shape[0] + 1, dtype=np.int64)
    crow[1:] = np.cumsum(keep.sum(axis=1))
    rows, cols = np.nonzero(keep)  # row-major: columns ascending inside each row
    return crow, cols.astype(np.int64), x[rows, cols]


def topk(reps, k: int):
    """(values [B, k], indices [B, k]) by value descending, then vocab id ascending."""
    x = np.asarray(reps, dtype=np.float64)
    B, V = x.shape
    key = np.where(np.isnan(x), np.inf, x)
    nan_first = np.isnan(x)
    vals = np.empty((B, k), dtype=np.asarray(reps).dtype)
    idx = np.empty((B, k), dtype=np.int64)
    for b in range(B):
        # lexsort: last key is primary. NaN first, then larger values, then lower ids.
        order = np.lexsort((np.arange(V), -key[b], ~nan_first[b]))[:k]
        idx[b] = order
        vals[b] = np.asarray(reps)[b, order]
    return vals, idx


def nonzero_ratio(reps) -> float:
    return float((np.asarray(reps) > 0).mean())
