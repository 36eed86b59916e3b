"""Generates the golden fixtures in this directory from the REFERENCE itself.

Runs hhkbble/sparton's own pure-PyTorch head, ``ProjectionPyTorch`` from
training/model.py:48-62 (the ``--head torch`` math), on the CPU with
``transform = nn.Identity()`` and ``decoder = nn.Linear(D, V)``, forward and
backward under autograd, on small seeded inputs. The outputs (reps and the
gradients of hidden, decoder weight and bias) are saved as ``<case>.npz``
together with the inputs, and pin the numpy oracle in ``oracle/`` before the
tests trust it.

This script needs a checkout of the reference (``--reference PATH``, the
project root of hhkbble/sparton), which exists only where the fixtures are made; the
fixtures themselves are committed and the tests never read the reference.

    python tests/golden/make_golden.py --reference PATH
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch
from torch import nn

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (dtype, B, S, D, V, lengths or "holes", use_bias, seed)
CASES = {
    "small_f64_bias": (torch.float64, 3, 37, 64, 300, [37, 20, 5], True, 1),
    "small_f64_nobias_emptyrow": (torch.float64, 4, 33, 32, 257, [33, 0, 1, 17], False, 2),
    "holes_f64": (torch.float64, 2, 20, 48, 130, "holes", True, 3),
    "cfg1like_f32": (torch.float32, 2, 24, 96, 500, [24, 9], True, 4),
    "small_bf16": (torch.bfloat16, 2, 40, 64, 200, [40, 13], True, 5),
    "small_f16": (torch.float16, 2, 40, 64, 200, [31, 40], True, 6),
}


def make_inputs(dtype, B, S, D, V, lengths, use_bias, seed):
    gen = torch.Generator().manual_seed(seed)
    H = torch.randn(B, S, D, generator=gen, dtype=torch.float64)
    W = torch.randn(V, D, generator=gen, dtype=torch.float64) * (0.5 / D ** 0.5)
    b = torch.randn(V, generator=gen, dtype=torch.float64) * 0.05 if use_bias else None
    if lengths == "holes":
        mask = (torch.rand(B, S, generator=gen) < 0.6).to(torch.int64)
    else:
        mask = torch.zeros(B, S, dtype=torch.int64)
        for i, L in enumerate(lengths):
            mask[i, :L] = 1
    g = torch.randn(B, V, generator=gen, dtype=torch.float64)
    cast = lambda t: None if t is None else t.to(dtype)
    return cast(H), cast(W), cast(b), mask, cast(g)


def run_reference(reference: str, H, W, b, mask, g):
    sys.path.insert(0, os.path.join(reference, "training"))
    from model import ProjectionPyTorch  # the reference's own head

    D, V = H.shape[2], W.shape[0]
    decoder = nn.Linear(D, V, bias=b is not None, dtype=H.dtype)
    with torch.no_grad():
        decoder.weight.copy_(W)
        if b is not None:
            decoder.bias.copy_(b)
    head = ProjectionPyTorch(nn.Identity(), decoder)
    hid = H.clone().requires_grad_(True)
    reps = head(hid, mask)
    reps.backward(g)
    return (reps.detach(), hid.grad.detach(), decoder.weight.grad.detach(),
            None if b is None else decoder.bias.grad.detach())


def as_np(t):
    return None if t is None else t.detach().to(torch.float64).numpy()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="project root of hhkbble/sparton")
    args = ap.parse_args()
    for name, spec in CASES.items():
        dtype = spec[0]
        H, W, b, mask, g = make_inputs(*spec)
        reps, dH, dW, db = run_reference(args.reference, H, W, b, mask, g)
        out = dict(dtype=str(dtype).replace("torch.", ""), H=as_np(H), W=as_np(W),
                   mask=mask.numpy(), g=as_np(g), reps=as_np(reps), dH=as_np(dH), dW=as_np(dW),
                   has_bias=np.array(b is not None))
        if b is not None:
            out.update(bias=as_np(b), db=as_np(db))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
        print(f"{name}: {dtype} B={H.shape[0]} S={H.shape[1]} D={H.shape[2]} V={W.shape[0]}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
