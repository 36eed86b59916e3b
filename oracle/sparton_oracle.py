"""CPU oracle for the SPLADE head — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module, and only as the checker / the timed CPU reference. The
product path (``sparton_b200``) never calls it and has no CPU fallback.

Restates, in float64 numpy, the math of hhkbble/sparton:

* the reference torch head (the "--head torch" path), training/model.py:56-62:
  ``reps = log1p(relu(logits * mask[..., None])).max(dim=1).values`` with
  ``logits = decoder(hidden) = hidden @ W.T + bias``;
* the argmax rule of the fused forward kernel, src/sparton/sparton_kernel.py:
  running max initialised to 0 with index 0 (:112-114), masked logits forced
  to 0 (:147-148), strict ``>`` between S-tiles and the first index inside a
  tile (:151-156), i.e. the smallest s attaining the max, 0 when max <= 0;
  then ``log(1 + relu(max))`` (:158-161);
* the fused backward kernel (:472-565): ``g' = where(score > 0,
  g * exp(-score), 0)`` (:531), ``db[v] = sum_b g'`` (:536),
  ``dW[v] = sum_b g' * H[b, idx[b, v]]`` (:554-557),
  ``dH[b, idx[b, v]] += g' * W[v]`` (:559-561).

Parity is pinned against fixtures produced by running the reference's own torch
head (tests/golden/make_golden.py); the test suite checks this module against
them before trusting it.
"""
from __future__ import annotations

import numpy as np

# Relative size, against sum_d |h_d * w_d|, of a logit difference treated as a
# near-tie. fp32 accumulation of D products has rounding error of order
# sqrt(D) * 2^-24 * sum|h*w| (worst case D * 2^-24); 2^-16 covers D <= 256 worst
# case and any practical D on average. Argmax indices must match exactly except
# where the top two candidates (or the max and 0) are closer than this.
NEAR_TIE_REL = 2.0 ** -16


def _f64(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float64)


def logits(H, W, bias=None) -> np.ndarray:
    """[B,S,V] float64 logits ``H @ W.T + bias`` (model.py:58, decoder)."""
    z = np.einsum("bsd,vd->bsv", _f64(H), _f64(W), optimize=True)
    if bias is not None:
        z = z + _f64(bias)[None, None, :]
    return z


def forward(H, W, bias, mask):
    """(reps[B,V], idx[B,V], max_logit[B,V]) in float64 / int64.

    reps = log1p(relu(max over valid s of logits)); idx = smallest s attaining a
    positive max, else 0. Invalid (mask 0) positions never win: they hold 0,
    which does not beat the initial 0 (sparton_kernel.py:112, :147-156)."""
    z = logits(H, W, bias)
    valid = _f64(mask) != 0
    zm = np.where(valid[:, :, None], z, -np.inf)
    m = zm.max(axis=1)
    first = zm.argmax(axis=1)  # first occurrence of the max
    pos = m > 0
    reps = np.where(pos, np.log1p(np.where(pos, m, 0.0)), 0.0)
    idx = np.where(pos, first, 0).astype(np.int64)
    return reps, idx, m


def near_tie_mask(H, W, bias, mask, rel: float = NEAR_TIE_REL):
    """[B,V] bool: entries whose argmax (or sign of the max) is within rounding
    of fp32 accumulation, i.e. top-2 valid logits, or the max and 0, closer than
    ``rel * sum_d |h_d w_d|`` of the top candidate."""
    z = logits(H, W, bias)
    valid = _f64(mask) != 0
    zm = np.where(valid[:, :, None], z, -np.inf)
    scale = np.einsum("bsd,vd->bsv", np.abs(_f64(H)), np.abs(_f64(W)), optimize=True)
    top = zm.argmax(axis=1)
    m = np.take_along_axis(zm, top[:, None, :], axis=1)[:, 0, :]
    sc = np.take_along_axis(scale, top[:, None, :], axis=1)[:, 0, :]
    tol = rel * (sc + (np.abs(_f64(bias))[None, :] if bias is not None else 0.0)) + 1e-30
    zs = np.sort(zm, axis=1)
    second = zs[:, -2, :] if zm.shape[1] > 1 else np.full_like(m, -np.inf)
    with np.errstate(invalid="ignore"):  # rows with no valid position: -inf - -inf
        tie = (m - second) <= tol
    sign = np.abs(m) <= tol
    return (tie | sign) & np.isfinite(m)


def accept_indices(idx_test, H, W, bias, mask, rel: float = NEAR_TIE_REL):
    """[B,V] bool: whether each tested argmax is acceptable. Exact match with
    the oracle is required outside near-ties; at a near-tie any valid position
    whose logit is within the tolerance of the max (or index 0 when the max is
    within tolerance of 0) is accepted."""
    reps, idx, m = forward(H, W, bias, mask)
    idx_test = np.asarray(idx_test, dtype=np.int64)
    ok = idx_test == idx
    near = near_tie_mask(H, W, bias, mask, rel)
    if near.any():
        z = logits(H, W, bias)
        valid = _f64(mask) != 0
        scale = np.einsum("bsd,vd->bsv", np.abs(_f64(H)), np.abs(_f64(W)), optimize=True)
        b_i, v_i = np.nonzero(near & ~ok)
        for b, v in zip(b_i, v_i):
            s = idx_test[b, v]
            mv = m[b, v]
            tol = rel * (scale[b, :, v].max() + (abs(float(bias[v])) if bias is not None else 0.0))
            if mv <= tol and s == 0:
                ok[b, v] = True  # max ~ 0: index 0 is the no-positive-logit answer
            elif 0 <= s < z.shape[1] and valid[b, s] and z[b, s, v] >= mv - tol and z[b, s, v] > -tol:
                ok[b, v] = True
    return ok


def backward_from_scores(g, scores, idx, H, W, has_bias: bool):
    """(dH[B,S,D], dW[V,D], db[V] or None) float64 from the forward's stored
    scores and indices, exactly as the fused backward kernel defines them
    (sparton_kernel.py:531-561)."""
    g = _f64(g)
    scores = _f64(scores)
    idx = np.asarray(idx, dtype=np.int64)
    H = _f64(H)
    W = _f64(W)
    B, S, D = H.shape
    V = W.shape[0]
    gp = np.where(scores > 0, g * np.exp(-scores), 0.0)
    db = gp.sum(axis=0) if has_bias else None
    dW = np.zeros((V, D))
    dH = np.zeros((B, S, D))
    for b in range(B):
        rows = H[b][idx[b]]  # [V, D] gathered argmax rows
        dW += gp[b][:, None] * rows
        P = np.zeros((S, V))
        P[idx[b], np.arange(V)] = gp[b]
        dH[b] = P @ W
    return dH, dW, db


def backward_exact(g, H, W, bias, mask):
    """(dH, dW, db or None) float64 of the torch head itself (model.py:56-62
    under autograd): the gradient reaches the argmax position only, scaled by
    d log1p(x)/dx = 1/(1+x) where the max logit x > 0."""
    g = _f64(g)
    reps, idx, m = forward(H, W, bias, mask)
    H = _f64(H)
    W = _f64(W)
    B, S, D = H.shape
    V = W.shape[0]
    gp = np.where(m > 0, g / (1.0 + np.where(m > 0, m, 0.0)), 0.0)
    db = gp.sum(axis=0) if bias is not None else None
    dW = np.zeros((V, D))
    dH = np.zeros((B, S, D))
    for b in range(B):
        dW += gp[b][:, None] * H[b][idx[b]]
        P = np.zeros((S, V))
        P[idx[b], np.arange(V)] = gp[b]
        dH[b] = P @ W
    return dH, dW, db


def sharded_backward_hidden(g_shards, score_shards, idx_shards, H, W_shards):
    """dH of a vocabulary-sharded head: the sum over shards of each shard's
    partial dH (what the all-reduce produces)."""
    total = None
    for g, sc, ix, Ws in zip(g_shards, score_shards, idx_shards, W_shards):
        dH, _, _ = backward_from_scores(g, sc, ix, H, Ws, False)
        total = dH if total is None else total + dH
    return total
