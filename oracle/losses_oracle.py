"""CPU oracle for the training losses that consume the head — TEST
INFRASTRUCTURE ONLY.

Only ``tests/`` and ``bench.py``'s CPU legs may import this module, and only as
the checker; the product path (``sparton_b200.losses``) never calls it.

Restates, in float64 numpy, hhkbble/sparton training/train.py:

* ``info_nce_loss`` (:73-77): ``scores = q @ d.T / temperature``, cross
  entropy against labels ``arange(Bq)`` (mean over queries);
* ``l1_regularization`` (:80-82): ``mean_b sum_v |reps[b, v]|``;
* ``flops_regularization`` (:85-87): ``mean_v (sum_b reps[b, v])^2``;

each with its gradient, and the vocab-sharded forms used by
``sparton_b200.losses`` (sums of per-shard partials). Pinned against fixtures
produced by running those reference functions under autograd
(tests/golden/make_golden_losses.py).
"""
from __future__ import annotations

import numpy as np


def _f64(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float64)


def info_nce(q, d, temperature: float = 1.0):
    """(loss, dloss/dq, dloss/dd)."""
    q, d = _f64(q), _f64(d)
    s = q @ d.T / temperature
    m = s.max(axis=1, keepdims=True)
    e = np.exp(s - m)
    p = e / e.sum(axis=1, keepdims=True)
    n = s.shape[0]
    loss = float(np.mean(np.log(e.sum(axis=1)) + m[:, 0] - s[np.arange(n), np.arange(n)]))
    ds = p.copy()
    ds[np.arange(n), np.arange(n)] -= 1.0
    ds /= n
    return loss, ds @ d / temperature, ds.T @ q / temperature


def l1(reps):
    """(value, dvalue/dreps); the gradient of |x| at 0 is 0, as in torch."""
    x = _f64(reps)
    return float(np.mean(np.abs(x).sum(axis=1))), np.sign(x) / x.shape[0]


def flops(reps):
    """(value, dvalue/dreps)."""
    x = _f64(reps)
    col = x.sum(axis=0)
    return float(np.mean(col ** 2)), np.broadcast_to(2.0 * col / x.shape[1], x.shape).copy()


def sharded_scores(q_shards, d_shards):
    """q @ d.T as the sum over vocabulary shards of the per-shard partials."""
    return sum(_f64(q) @ _f64(d).T for q, d in zip(q_shards, d_shards))
