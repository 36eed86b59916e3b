"""Generates the sparse-form fixtures in this directory with torch, the
reference's own dependency for these conversions (hhkbble/sparton
pyproject.toml: torch>=2.7.1; its encode, training/model.py:141-144, returns
dense reps and train.py:205-210 measures (reps > 0).float().mean()).

For seeded SPLADE-like reps (log1p(relu(x)): non-negative, many exact zeros,
16-bit rounding ties) plus signed and NaN cases, saves ``sparse_<case>.npz``:
reps (as float32, exact for the 16-bit dtypes), the threshold, the CSR arrays
of the entries ``reps > threshold`` in row-major order (checked equal to
``reps.to_sparse_csr()`` for threshold 0 on non-negative reps), the values of
``torch.topk(reps, k, dim=1)`` for a few k, and ``(reps > 0).float().mean()``.
They pin oracle/sparse_oracle.py before the tests trust it.

    python tests/golden/make_golden_sparse.py
"""
from __future__ import annotations

import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (dtype, B, V, zero fraction, threshold, signed, nan, seed, ks)
CASES = {
    "sparse_bf16": (torch.bfloat16, 6, 1000, 0.6, 0.0, False, False, 21, (1, 7, 64, 1000)),
    "sparse_f16_thr": (torch.float16, 4, 4099, 0.3, 0.5, False, False, 22, (3, 100, 4096)),
    "sparse_f32_signed_nan": (torch.float32, 3, 300, 0.2, -0.25, True, True, 23, (1, 5, 300)),
}


def make(dtype, B, V, zero_frac, thr, signed, nan, seed, ks):
    gen = torch.Generator().manual_seed(seed)
    x = torch.log1p(torch.relu(torch.randn(B, V, generator=gen) * 2.0))
    x[torch.rand(B, V, generator=gen) < zero_frac] = 0.0
    if signed:
        x = x - 0.5 * torch.rand(B, V, generator=gen)
    if nan:
        x[0, 7] = float("nan")
        x[1, 3] = float("inf")
    reps = x.to(dtype)
    keep = reps > thr
    crow = torch.zeros(B + 1, dtype=torch.int64)
    crow[1:] = keep.sum(dim=1).cumsum(0)
    cols = keep.nonzero()[:, 1]  # row-major order
    vals = reps[keep]
    if thr == 0.0 and not signed:  # the head's non-negative output: to_sparse_csr itself
        c = reps.to_sparse_csr()
        assert torch.equal(c.crow_indices(), crow) and torch.equal(c.col_indices(), cols)
        assert torch.equal(c.values(), vals)
    out = {
        "dtype": str(dtype).split(".")[-1], "reps": reps.float().numpy(), "threshold": thr,
        "crow": crow.numpy(), "cols": cols.numpy(), "vals": vals.float().numpy(),
        "ks": np.array(ks),
        "nonzero_ratio": float((reps > 0).float().mean()),
    }
    for k in ks:
        v, _ = torch.topk(reps, k, dim=1)
        out[f"topk{k}"] = v.float().numpy()
    return out


def main() -> None:
    for name, spec in CASES.items():
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **make(*spec))
        print("wrote", name)


if __name__ == "__main__":
    main()
