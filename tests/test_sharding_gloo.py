"""Vocabulary-sharded SpartonHead on 2 CPU ranks (gloo): shard bounds, the forward
without communication, the optional all-gather of reps, and the all-reduce of
the partial d_hidden in the backward. The native operators are replaced inside
the test by CPU stand-ins computed with the oracle, so what is tested is the
host logic of the sharded path (partitioning, autograd wiring, collectives)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import sparton_oracle as orc
from sparton_b200 import head as head_mod
from sparton_b200 import ops
from sparton_b200.head import SpartonHead, VocabShard

B, S, D, V = 3, 11, 16, 300


def _inputs():
    gen = torch.Generator().manual_seed(7)
    H = torch.randn(B, S, D, generator=gen, dtype=torch.float64)
    W = torch.randn(V, D, generator=gen, dtype=torch.float64) * 0.3
    b = torch.randn(V, generator=gen, dtype=torch.float64) * 0.05
    L = torch.tensor([11, 4, 0])
    mask = (torch.arange(S)[None, :] < L[:, None]).to(torch.int64)
    g = torch.randn(B, V, generator=gen, dtype=torch.float64)
    return H, W, b, mask, g


def _cpu_forward(hidden, embed, bias, mask):
    reps, idx, _ = orc.forward(hidden.detach().numpy(), embed.detach().numpy(),
                               None if bias is None else bias.detach().numpy(), mask.numpy())
    return torch.tensor(reps, dtype=hidden.dtype), torch.tensor(idx, dtype=torch.int32)


def _cpu_backward(grad_out, scores, idx, hidden, embed, has_bias, need_hidden=True,
                  need_embed=True, hidden_grad_dtype=None):
    dH, dW, db = orc.backward_from_scores(grad_out.numpy(), scores.numpy(), idx.numpy(),
                                          hidden.detach().numpy(), embed.detach().numpy(), has_bias)
    gdt = hidden_grad_dtype or hidden.dtype
    return (torch.tensor(dH, dtype=gdt) if need_hidden else None,
            torch.tensor(dW, dtype=embed.dtype) if need_embed else None,
            torch.tensor(db, dtype=embed.dtype) if has_bias else None)


def _cpu_hidden_rows(grad_out, scores, idx, hidden, embed, out, b0, b1, workspace=None):
    dH, _, _ = orc.backward_from_scores(grad_out[b0:b1].numpy(), scores[b0:b1].numpy(),
                                        idx[b0:b1].numpy(), hidden[b0:b1].detach().numpy(),
                                        embed.detach().numpy(), False)
    out[b0:b1] = torch.tensor(dH, dtype=out.dtype)


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ops.forward_impl = _cpu_forward
        ops.backward_impl = _cpu_backward
        ops.hidden_grad_rows = _cpu_hidden_rows
        H, W, b, mask, g = _inputs()
        for gather in (False, True):
            # gather_output=True also runs the d_hidden all-reduce one batch row
            # per chunk (one collective per chunk, all in flight together).
            head_mod.REDUCE_CHUNK_BYTES = 1 if gather else 128 << 20
            head = SpartonHead(V, D, use_bias=True, process_group=dist.group.WORLD,
                               gather_output=gather).double()
            head.load({"weight": W, "bias": b})
            sh = head.shard
            hid = H.clone().requires_grad_(True)
            reps = head(hid, mask)
            if gather:
                assert reps.shape == (B, V)
                reps.backward(g)
            else:
                assert reps.shape == (B, sh.size)
                reps.backward(g[:, sh.start:sh.stop])
            np.save(os.path.join(out_dir, f"r{rank}_g{int(gather)}_reps.npy"), reps.detach().numpy())
            np.save(os.path.join(out_dir, f"r{rank}_g{int(gather)}_dH.npy"), hid.grad.numpy())
            np.save(os.path.join(out_dir, f"r{rank}_g{int(gather)}_dW.npy"), head.weight.grad.numpy())
            np.save(os.path.join(out_dir, f"r{rank}_g{int(gather)}_db.npy"), head.bias.grad.numpy())
            np.save(os.path.join(out_dir, f"r{rank}_shard.npy"), np.array([sh.start, sh.stop]))
        # float32 hidden states with a float64 reduce dtype: reduce-scatter in
        # float64, parts rounded to float32, all-gather (one chunk, then one
        # batch row per chunk).
        head_mod.REDUCE_SCATTER_GATHER = True
        for chunk in (128 << 20, 1):
            head_mod.REDUCE_CHUNK_BYTES = chunk
            head = SpartonHead(V, D, use_bias=True, process_group=dist.group.WORLD,
                               grad_reduce_dtype=torch.float64).float()
            head.load({"weight": W.float(), "bias": b.float()})
            sh = head.shard
            hid = H.float().clone().requires_grad_(True)
            reps = head(hid, mask)
            reps.backward(g[:, sh.start:sh.stop].float())
            assert hid.grad.dtype == torch.float32
            np.save(os.path.join(out_dir, f"r{rank}_rs{int(chunk == 1)}_dH.npy"), hid.grad.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_vocab_shard_bounds():
    for world in (1, 2, 3, 4, 8):
        shards = [VocabShard(30522, world, r) for r in range(world)]
        assert shards[0].start == 0 and shards[-1].stop == 30522
        for a, c in zip(shards, shards[1:]):
            assert a.stop == c.start
        if world > 1:
            assert all(s.padded % head_mod.VOCAB_TILE == 0 for s in shards)
    tiny = [VocabShard(100, 4, r) for r in range(4)]  # more ranks than tiles: empty shards
    assert [t.size for t in tiny] == [100, 0, 0, 0]


def test_row_chunks():
    assert head_mod.row_chunks(128, 256 * 768 * 4) == [(0, 128)]  # 100 MB: one chunk
    c = head_mod.row_chunks(64, 1024 * 4096 * 4)  # 1 GB: 8 chunks of 8 rows
    assert c == [(8 * i, 8 * i + 8) for i in range(8)]
    c = head_mod.row_chunks(3, 10, chunk_bytes=1)
    assert c == [(0, 1), (1, 2), (2, 3)]
    c = head_mod.row_chunks(5, 1 << 30)
    assert c[0][0] == 0 and c[-1][1] == 5 and all(a < b for a, b in c)
    assert all(p[1] == q[0] for p, q in zip(c, c[1:]))


def test_sharded_head_two_ranks(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    H, W, b, mask, g = _inputs()
    reps, idx, _ = orc.forward(H.numpy(), W.numpy(), b.numpy(), mask.numpy())
    dH, dW, db = orc.backward_from_scores(g.numpy(), reps, idx, H.numpy(), W.numpy(), True)
    for gather in (0, 1):
        for r in range(world):
            lo, hi = np.load(tmp_path / f"r{r}_shard.npy")
            got = np.load(tmp_path / f"r{r}_g{gather}_reps.npy")
            np.testing.assert_allclose(got, reps if gather else reps[:, lo:hi], rtol=1e-12)
            # every rank holds the full d_hidden after the all-reduce
            np.testing.assert_allclose(np.load(tmp_path / f"r{r}_g{gather}_dH.npy"), dH,
                                       rtol=1e-10, atol=1e-12)
            np.testing.assert_allclose(np.load(tmp_path / f"r{r}_g{gather}_dW.npy"), dW[lo:hi],
                                       rtol=1e-10, atol=1e-12)
            np.testing.assert_allclose(np.load(tmp_path / f"r{r}_g{gather}_db.npy"), db[lo:hi],
                                       rtol=1e-10, atol=1e-12)
    # reduce-scatter path: float32 hidden states, float32 inputs to the oracle
    H32, W32, b32, g32 = (t.float().double() for t in (H, W, b, g))
    reps32, idx32, _ = orc.forward(H32.numpy(), W32.numpy(), b32.numpy(), mask.numpy())
    dH32, _, _ = orc.backward_from_scores(g32.numpy(), reps32.astype(np.float32), idx32,
                                          H32.numpy(), W32.numpy(), True)
    for rows in (0, 1):
        for r in range(world):
            np.testing.assert_allclose(np.load(tmp_path / f"r{r}_rs{rows}_dH.npy"), dH32,
                                       rtol=1e-5, atol=1e-6)


def _tie_worker(rank, world, port, out_dir):
    """Sharded tie_weights: the head trains this rank's rows of the decoder's
    storage with a shard-sized gradient; gather_weights assembles the full
    tensors after each rank updated its rows."""
    from torch import nn

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ops.forward_impl = _cpu_forward
        ops.backward_impl = _cpu_backward
        ops.hidden_grad_rows = _cpu_hidden_rows
        H, W, b, mask, g = _inputs()
        decoder = nn.Linear(D, V).double()
        with torch.no_grad():
            decoder.weight.copy_(W)
            decoder.bias.copy_(b)
        head = SpartonHead(V, D, use_bias=True, process_group=dist.group.WORLD).double()
        head.tie_weights(decoder)
        sh = head.shard
        assert head.weight.shape == (sh.size, D) and head.bias.shape == (sh.size,)
        assert head.weight.data_ptr() == decoder.weight[sh.start].data_ptr()
        hid = H.clone().requires_grad_(True)
        head(hid, mask).backward(g[:, sh.start:sh.stop])
        assert head.weight.grad.shape == (sh.size, D)  # shard-sized, not [V, D]
        assert decoder.weight.grad is None
        with torch.no_grad():  # an optimizer step on the shard lands in the decoder's rows
            head.weight.add_(1.0)
            head.bias.add_(1.0)
        assert torch.equal(decoder.weight[sh.start:sh.stop], W[sh.start:sh.stop] + 1.0)
        full_w, full_b = head.gather_weights(out_weight=decoder.weight.data,
                                             out_bias=decoder.bias.data)
        np.save(os.path.join(out_dir, f"tie_r{rank}_w.npy"), full_w.numpy())
        np.save(os.path.join(out_dir, f"tie_r{rank}_b.npy"), full_b.numpy())
        np.save(os.path.join(out_dir, f"tie_r{rank}_dW.npy"), head.weight.grad.numpy())
        np.save(os.path.join(out_dir, f"tie_r{rank}_shard.npy"), np.array([sh.start, sh.stop]))
    finally:
        dist.destroy_process_group()


def test_sharded_tie_weights_keeps_shard_sized_grads(tmp_path):
    world = 2
    mp.start_processes(_tie_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    H, W, b, mask, g = _inputs()
    reps, idx, _ = orc.forward(H.numpy(), W.numpy(), b.numpy(), mask.numpy())
    _, dW, _ = orc.backward_from_scores(g.numpy(), reps, idx, H.numpy(), W.numpy(), True)
    for r in range(world):
        lo, hi = np.load(tmp_path / f"tie_r{r}_shard.npy")
        np.testing.assert_allclose(np.load(tmp_path / f"tie_r{r}_dW.npy"), dW[lo:hi], rtol=1e-10,
                                   atol=1e-12)
        # every rank added 1 to its own rows: the gathered tensors are W + 1 everywhere
        np.testing.assert_allclose(np.load(tmp_path / f"tie_r{r}_w.npy"), W.numpy() + 1.0,
                                   rtol=0, atol=0)
        np.testing.assert_allclose(np.load(tmp_path / f"tie_r{r}_b.npy"), b.numpy() + 1.0,
                                   rtol=0, atol=0)
