"""CPU oracle for the MLM transform in front of the head — TEST
INFRASTRUCTURE ONLY.

Only ``tests/`` and ``bench.py``'s CPU legs may import this module, and only as
the checker; the product path (``sparton_b200.transform``) never calls it.

Restates, in float64 numpy, hhkbble/sparton training/model.py:25-35 (the
RoBERTa transform: dense, ``transformers.activations.gelu`` = exact erf gelu,
LayerNorm; BERT's ``predictions.transform`` is the same three layers) and the
projection ``ProjectionPyTorch`` (:48-62) that feeds it to the head, with the
gradients of every input and parameter. Pinned against fixtures made by
running the reference's own ``_get_backbone_and_head`` and ``ProjectionPyTorch``
on small random-init BERT and RoBERTa masked-LM models
(tests/golden/make_golden_transform.py).
"""
from __future__ import annotations

import numpy as np
from scipy.special import erf

from oracle import sparton_oracle as orc

_SQRT1_2 = 0.7071067811865476
_INV_SQRT_2PI = 0.3989422804014327


def _f64(x):
    return np.asarray(x, dtype=np.float64)


def round_to(a, dtype: str):
    """float64 values rounded to `dtype` ("float64", "float32", "float16",
    "bfloat16"; round to nearest even), as float64."""
    a = _f64(a)
    if dtype == "float64":
        return a
    if dtype == "float16":
        return a.astype(np.float16).astype(np.float64)
    a32 = a.astype(np.float32)
    if dtype == "float32":
        return a32.astype(np.float64)
    u = a32.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return u.view(np.float32).astype(np.float64)


def gelu(y, act_dtype: str = "float64"):
    """Exact erf gelu, rounded to `act_dtype` as a separate activation module
    in that dtype rounds its output."""
    y = _f64(y)
    return round_to(0.5 * y * (1.0 + erf(y * _SQRT1_2)), act_dtype)


def transform_forward(x, Wd, bd, gamma, beta, eps, act_dtype: str = "float64"):
    """(h, cache): h = LayerNorm(gelu(x @ Wd^T + bd)) * gamma + beta."""
    x, Wd, gamma, beta = _f64(x), _f64(Wd), _f64(gamma), _f64(beta)
    y = x @ Wd.T + (0.0 if bd is None else _f64(bd))
    return layer_norm_gelu(y, gamma, beta, eps, act_dtype, x, Wd)


def layer_norm_gelu(y, gamma, beta, eps, act_dtype: str = "float64", x=None, Wd=None):
    """(h, cache) of the gelu + LayerNorm part alone, from y."""
    y, gamma, beta = _f64(y), _f64(gamma), _f64(beta)
    g = gelu(y, act_dtype)
    mu = g.mean(axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt(((g - mu) ** 2).mean(axis=-1, keepdims=True) + eps)
    xh = (g - mu) * rstd
    return xh * gamma + beta, (x, Wd, gamma, y, rstd, xh)


def transform_backward(dh, cache):
    """(dx, dWd, dbd, dgamma, dbeta) from dh = dLoss/dh."""
    x, Wd, gamma, y, rstd, xh = cache
    dy, dgamma, dbeta = layer_norm_gelu_backward(dh, cache)
    D = y.shape[-1]
    flat = lambda t: t.reshape(-1, t.shape[-1])  # noqa: E731
    dx = dy @ Wd
    dWd = flat(dy).T @ flat(x)
    dbd = flat(dy).sum(axis=0)
    assert dWd.shape == (D, x.shape[-1])
    return dx, dWd, dbd, dgamma, dbeta


def layer_norm_gelu_backward(dh, cache):
    """(dy, dgamma, dbeta) of the gelu + LayerNorm part."""
    _, _, gamma, y, rstd, xh = cache
    dh = _f64(dh)
    flat = lambda t: t.reshape(-1, t.shape[-1])  # noqa: E731
    dgamma = (flat(dh) * flat(xh)).sum(axis=0)
    dbeta = flat(dh).sum(axis=0)
    dxh = dh * gamma
    dg = rstd * (dxh - dxh.mean(axis=-1, keepdims=True)
                 - xh * (dxh * xh).mean(axis=-1, keepdims=True))
    dy = dg * (0.5 * (1.0 + erf(y * _SQRT1_2)) + y * _INV_SQRT_2PI * np.exp(-0.5 * y * y))
    return dy, dgamma, dbeta


def projection(x, Wd, bd, gamma, beta, eps, W, b, mask, g):
    """ProjectionPyTorch(transform, decoder) forward and backward in float64:
    (reps, grads) with grads = dict of dx, dWd, dbd, dgamma, dbeta, dW, db."""
    h, cache = transform_forward(x, Wd, bd, gamma, beta, eps)
    reps, _, _ = orc.forward(h, W, b, mask)
    dh, dW, db = orc.backward_exact(g, h, W, b, mask)
    dx, dWd, dbd, dgamma, dbeta = transform_backward(dh, cache)
    return reps, dict(dx=dx, dWd=dWd, dbd=dbd, dgamma=dgamma, dbeta=dbeta, dW=dW, db=db), h
