"""Generates the loss fixtures in this directory from the REFERENCE itself.

Runs hhkbble/sparton's own training losses, ``info_nce_loss``,
``l1_regularization`` and ``flops_regularization`` from training/train.py:73-87,
on the CPU under autograd, on small seeded SPLADE-like representations
(non-negative, many exact zeros). Saves inputs, loss values and the gradients
with respect to the query / document representations as ``losses_<case>.npz``;
they pin the loss oracle in ``oracle/losses_oracle.py`` before the tests trust
it.

This script needs a checkout of the reference (``--reference PATH``, the
project root of hhkbble/sparton), which exists only where the fixtures are made; the
fixtures themselves are committed and the tests never read the reference.

    python tests/golden/make_golden_losses.py --reference PATH
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (dtype, Bq, Bd, V, temperature, zero fraction, seed)
CASES = {
    "losses_f64": (torch.float64, 6, 6, 300, 1.0, 0.5, 11),
    "losses_f32_temp": (torch.float32, 8, 8, 1000, 0.05, 0.9, 12),
    "losses_bf16": (torch.bfloat16, 4, 4, 257, 1.0, 0.3, 13),
}


def load_reference_train(reference: str):
    sys.path.insert(0, os.path.join(reference, "training"))
    spec = importlib.util.spec_from_file_location(
        "reference_train", os.path.join(reference, "training", "train.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_reps(B, V, zero_frac, gen):
    x = torch.rand(B, V, generator=gen, dtype=torch.float64) * 2.0
    x[torch.rand(B, V, generator=gen) < zero_frac] = 0.0
    return x


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="project root of hhkbble/sparton")
    args = ap.parse_args(argv)
    ref = load_reference_train(args.reference)
    for name, (dtype, Bq, Bd, V, temp, zf, seed) in CASES.items():
        gen = torch.Generator().manual_seed(seed)
        q = make_reps(Bq, V, zf, gen).to(dtype).requires_grad_(True)
        d = make_reps(Bd, V, zf, gen).to(dtype).requires_grad_(True)
        out = {"q": q.detach().double().numpy(), "d": d.detach().double().numpy(),
               "temperature": np.float64(temp), "dtype": str(dtype).split(".")[-1]}
        nce = ref.info_nce_loss(q, d, temperature=temp)
        gq, gd = torch.autograd.grad(nce, (q, d))
        out.update(nce=np.float64(nce.item()), nce_dq=gq.double().numpy(), nce_dd=gd.double().numpy())
        l1 = ref.l1_regularization(q)
        (g1,) = torch.autograd.grad(l1, (q,))
        out.update(l1=np.float64(l1.item()), l1_dq=g1.double().numpy())
        fl = ref.flops_regularization(q)
        (gf,) = torch.autograd.grad(fl, (q,))
        out.update(flops=np.float64(fl.item()), flops_dq=gf.double().numpy())
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print(name, "nce", out["nce"], "l1", out["l1"], "flops", out["flops"])
    return 0


if __name__ == "__main__":
    sys.exit(main())
