"""Generates the MLM-transform fixtures in this directory from the REFERENCE
itself.

Builds small random-init BERT and RoBERTa masked-LM models with transformers
(no download: a config and seeded initialisation), extracts their transform and
decoder with the reference's own ``_get_backbone_and_head``
(training/model.py:7-45) and runs its ``ProjectionPyTorch`` (:48-62) in float64
on the CPU under autograd, on seeded hidden states, masks and upstream
gradients. Saves inputs, parameters, reps and every gradient as
``transform_<case>.npz``; they pin oracle/transform_oracle.py.

This script needs a checkout of the reference (``--reference PATH``, the
project root of hhkbble/sparton), which exists only where the fixtures are made; the
fixtures themselves are committed and the tests never read the reference.

    python tests/golden/make_golden_transform.py --reference PATH
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (model_type, B, S, D, V, seed)
CASES = {"transform_bert": ("bert", 3, 12, 32, 120, 31),
         "transform_roberta": ("roberta", 2, 9, 48, 90, 32)}


def build(model_type, D, V, seed):
    from transformers import BertConfig, BertForMaskedLM, RobertaConfig, RobertaForMaskedLM

    torch.manual_seed(seed)
    common = dict(vocab_size=V, hidden_size=D, num_hidden_layers=1, num_attention_heads=2,
                  intermediate_size=2 * D, max_position_embeddings=64)
    if model_type == "bert":
        llm = BertForMaskedLM(BertConfig(**common))
    else:
        llm = RobertaForMaskedLM(RobertaConfig(**common, pad_token_id=1))
    llm = llm.double()
    with torch.no_grad():  # non-trivial LayerNorm affine parameters and decoder bias
        for p in llm.parameters():
            if p.dim() == 1:
                p.add_(0.1 * torch.randn_like(p))
    return llm


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="project root of hhkbble/sparton")
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.reference, "training"))
    from model import ProjectionPyTorch, _get_backbone_and_head  # the reference's own

    for name, (mt, B, S, D, V, seed) in CASES.items():
        llm = build(mt, D, V, seed)
        _, transform, decoder = _get_backbone_and_head(llm)
        proj = ProjectionPyTorch(transform, decoder)
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn(B, S, D, generator=gen, dtype=torch.float64).requires_grad_(True)
        L = torch.randint(1, S + 1, (B,), generator=gen)
        L[-1] = 0 if B > 2 else L[-1]  # an empty row
        mask = (torch.arange(S)[None, :] < L[:, None]).to(torch.int64)
        g = torch.randn(B, V, generator=gen, dtype=torch.float64)
        reps = proj(x, mask)
        reps.backward(g)
        dense = transform.dense
        ln = transform.LayerNorm if hasattr(transform, "LayerNorm") else transform.layer_norm
        t = lambda p: p.detach().numpy()  # noqa: E731
        np.savez_compressed(
            os.path.join(HERE, f"{name}.npz"), x=t(x), mask=mask.numpy(), g=g.numpy(),
            Wd=t(dense.weight), bd=t(dense.bias), gamma=t(ln.weight), beta=t(ln.bias),
            eps=float(ln.eps), W=t(decoder.weight), b=t(decoder.bias), reps=t(reps),
            dx=t(x.grad), dWd=t(dense.weight.grad), dbd=t(dense.bias.grad),
            dgamma=t(ln.weight.grad), dbeta=t(ln.bias.grad), dW=t(decoder.weight.grad),
            db=t(decoder.bias.grad))
        print("wrote", name)


if __name__ == "__main__":
    main()
