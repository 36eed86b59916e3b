"""Shared input builders for the tests: golden fixtures and seeded synthetic
inputs with the value distributions of the benchmark configurations
(hidden ~ N(0,1), W ~ N(0, w_std), bias ~ N(0, 0.02), right-padded masks with
lengths uniform in a range, upstream grad g ~ N(0,1))."""
from __future__ import annotations

import glob
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

DTYPES = {"float64": torch.float64, "float32": torch.float32, "bfloat16": torch.bfloat16,
          "float16": torch.float16}


def golden_names():
    """The head's fixtures (the loss, sparse-form and transform fixtures,
    losses_*.npz, sparse_*.npz and transform_*.npz, have their own tests)."""
    return sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))
                  if not os.path.basename(p).startswith(("losses_", "sparse_", "transform_")))


def load_golden(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    d = {k: z[k] for k in z.files}
    d["dtype"] = str(d["dtype"])
    d["has_bias"] = bool(d["has_bias"])
    d.setdefault("bias", None)
    d.setdefault("db", None)
    return d


def synthetic(B, S, D, V, lengths=(1, None), dtype=torch.bfloat16, use_bias=True, w_std=0.02,
              seed=0, full_frac=0.0, holes=False):
    """CPU tensors (H, W, bias, mask int64, g) drawn like the benchmark configs.

    lengths: (lo, hi) inclusive range of valid lengths (hi None -> S).
    full_frac: fraction of rows forced to full length (config 4 uses 0.1)."""
    gen = torch.Generator().manual_seed(seed)
    H = torch.randn(B, S, D, generator=gen).to(dtype)
    W = (torch.randn(V, D, generator=gen) * w_std).to(dtype)
    b = (torch.randn(V, generator=gen) * 0.02).to(dtype) if use_bias else None
    lo, hi = lengths
    hi = S if hi is None else hi
    L = torch.randint(lo, hi + 1, (B,), generator=gen)
    if full_frac > 0:
        full = torch.rand(B, generator=gen) < full_frac
        L = torch.where(full, torch.full_like(L, S), L)
    mask = (torch.arange(S)[None, :] < L[:, None]).to(torch.int64)
    if holes:
        mask = mask * (torch.rand(B, S, generator=gen) < 0.7).to(torch.int64)
    g = torch.randn(B, V, generator=gen).to(dtype)
    return H, W, b, mask, g


def np64(t):
    return None if t is None else t.detach().to(torch.float64).cpu().numpy()
