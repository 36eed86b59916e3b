"""Vocabulary-sharded training losses (sparton_b200.losses) on 2 CPU ranks
(gloo): each rank holds one vocabulary shard of the query / document
representations; the InfoNCE scores are the all-reduced sum of per-shard
partials and the regularisers the all-reduced sum of per-shard totals. The two
native regulariser calls are replaced inside the test by CPU stand-ins, so what
is tested is the host logic (partials, collectives, autograd), against the
unsharded oracle."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import losses_oracle as lo
from sparton_b200 import losses

B, V, TEMP = 5, 301, 0.7
CUT = 160  # rank 0 owns columns [0, 160), rank 1 [160, 301)


def _inputs():
    gen = torch.Generator().manual_seed(3)
    q = torch.rand(B, V, generator=gen, dtype=torch.float64)
    d = torch.rand(B, V, generator=gen, dtype=torch.float64)
    q[q < 0.4] = 0.0
    d[d < 0.5] = 0.0
    return q, d


def _cpu_reg_forward(reps, scale_l1, scale_flops):
    x = reps.detach().double()
    col = x.sum(0)
    return col.float(), torch.stack([x.abs().sum() * scale_l1, (col ** 2).sum() * scale_flops]).float()


def _cpu_reg_backward(reps, colsum, g, scale_l1, scale_flops):
    g = g.double()
    return (g[0] * scale_l1 * torch.sign(reps.detach().double())
            + g[1] * scale_flops * colsum.double()[None, :]).to(reps.dtype)


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        losses.reg_forward_impl = _cpu_reg_forward
        losses.reg_backward_impl = _cpu_reg_backward
        q, d = _inputs()
        lo_, hi = (0, CUT) if rank == 0 else (CUT, V)
        qs = q[:, lo_:hi].clone().requires_grad_(True)
        ds = d[:, lo_:hi].clone().requires_grad_(True)
        g = dist.group.WORLD
        nce = losses.info_nce_loss(qs, ds, TEMP, process_group=g)
        l1, fl = losses.regularizers(qs, process_group=g, vocab_size=V)
        fl2 = losses.flops_regularization(qs, process_group=g)  # vocab size summed over ranks
        (nce + 0.3 * l1 + 0.2 * fl).backward()
        np.save(os.path.join(out_dir, f"r{rank}.npy"),
                np.array([nce.item(), l1.item(), fl.item(), fl2.item()]))
        np.save(os.path.join(out_dir, f"r{rank}_gq.npy"), qs.grad.numpy())
        np.save(os.path.join(out_dir, f"r{rank}_gd.npy"), ds.grad.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_losses_two_ranks(tmp_path):
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    q, d = _inputs()
    nce, dq, dd = lo.info_nce(q.numpy(), d.numpy(), TEMP)
    l1, g1 = lo.l1(q.numpy())
    fl, gf = lo.flops(q.numpy())
    want_gq = dq + 0.3 * g1 + 0.2 * gf
    for r, (a, b) in enumerate(((0, CUT), (CUT, V))):
        vals = np.load(tmp_path / f"r{r}.npy")
        np.testing.assert_allclose(vals, [nce, l1, fl, fl], rtol=1e-6)  # fp32 scores and totals
        # fp32 scores / totals: entries where terms of size ~1 cancel keep an
        # absolute error of a few fp32 ulps of those terms.
        np.testing.assert_allclose(np.load(tmp_path / f"r{r}_gq.npy"), want_gq[:, a:b], rtol=1e-5,
                                   atol=1e-6)
        np.testing.assert_allclose(np.load(tmp_path / f"r{r}_gd.npy"), dd[:, a:b], rtol=1e-5,
                                   atol=1e-6)
