"""Reference torch head on the CPU — TEST / BASELINE INFRASTRUCTURE ONLY.

Restates hhkbble/sparton's pure-PyTorch SPLADE head, training/model.py:56-62
(``ProjectionPyTorch.forward`` with ``transform = Identity``): the full
[B,S,V] logits through the decoder, ``log1p(relu(logits * mask))`` and a max
over the sequence, trained by plain autograd. It is what ``--head torch``
computes, and here it is the timed CPU baseline of ``bench.py`` (kind "port":
the reference cannot travel to the GPU box) and a cross-check in the tests.
Only tests, smoke() and bench.py's baseline legs use it.
"""
from __future__ import annotations

import os
import time

import torch


def torch_head(hidden: torch.Tensor, weight: torch.Tensor, bias, mask: torch.Tensor) -> torch.Tensor:
    """reps[B,V] = max_s log1p(relu((hidden @ weight.T + bias) * mask))  (model.py:58-61)."""
    logits = torch.nn.functional.linear(hidden, weight, bias)
    return torch.log1p(torch.relu(logits * mask.unsqueeze(-1).to(logits.dtype))).max(dim=1).values


def time_fwd_bwd(B: int, S: int, D: int, V: int, lengths, use_bias: bool = True, steps: int = 3,
                 warmup: int = 1, threads: int | None = None, seed: int = 0,
                 dtype: torch.dtype = torch.float32, w_std: float = 0.02) -> dict:
    """Times fwd+bwd of the torch head on the host (fp32 by default, every
    host thread). Returns seconds per step and the thread count used."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(seed)
    H = torch.randn(B, S, D, generator=gen, dtype=dtype).requires_grad_(True)
    W = (torch.randn(V, D, generator=gen) * w_std).to(dtype).requires_grad_(True)
    b = (torch.randn(V, generator=gen) * 0.02).to(dtype).requires_grad_(True) if use_bias else None
    mask = torch.zeros(B, S, dtype=torch.int64)
    for i, L in enumerate(lengths):
        mask[i, : int(L)] = 1
    g = torch.randn(B, V, generator=gen, dtype=dtype)
    times = []
    for it in range(warmup + steps):
        for p in (H, W, b):
            if p is not None:
                p.grad = None
        t0 = time.perf_counter()
        reps = torch_head(H, W, b, mask)
        reps.backward(g)
        dt = time.perf_counter() - t0
        if it >= warmup:
            times.append(dt)
    return {"seconds_per_step": sum(times) / len(times), "threads": threads, "steps": steps}
