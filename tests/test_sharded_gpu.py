"""Vocabulary-sharded SpartonHead on 2 and 4 GPUs (NCCL), against the same head
on one GPU: the forward shards and the d_weight / d_bias shards are
bit-identical (every vocab column is computed by the same kernel arithmetic
whichever rank owns it); d_hidden, an all-reduce of fp32 partial sums, matches
within one bf16 rounding (rtol 1e-2) plus 1e-2 of its largest entry. Run with
the all-reduce in one chunk, with one batch row per chunk, and with the head
tied to a full nn.Linear decoder (tie_weights: shard-sized gradients that land
in the decoder's rows). V = 3001 leaves a ragged last shard at every world
size. Both ways of summing the partial d_hidden run: over NVLink peer memory
(packed rows only, sparton_hidden_allreduce) and NCCL's all-reduce (in one
chunk and one batch row per chunk). Skipped with fewer GPUs than ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests._cases import synthetic

pytestmark = pytest.mark.gpu

B, S, D, V = 6, 160, 256, 3001


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir, reduce):
    import datetime

    from sparton_b200 import head as head_mod
    from sparton_b200.head import SpartonHead

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        H, W, b, mask, g = synthetic(B, S, D, V, (20, S), dtype=torch.bfloat16, seed=5,
                                     w_std=0.06)
        head_mod.HIDDEN_REDUCE = reduce
        for tag, chunk in (("one", 128 << 20), ("rows", 1), ("tied", 128 << 20)):
            head_mod.REDUCE_CHUNK_BYTES = chunk
            head = SpartonHead(V, D, use_bias=True, process_group=dist.group.WORLD).to(
                dev, torch.bfloat16)
            sh = head.shard
            if tag == "tied":
                decoder = torch.nn.Linear(D, V).to(dev, torch.bfloat16)
                with torch.no_grad():
                    decoder.weight.copy_(W)
                    decoder.bias.copy_(b)
                head.tie_weights(decoder)
                assert head.weight.shape == (sh.size, D)
            else:
                head.load({"weight": W[sh.start:sh.stop], "bias": b[sh.start:sh.stop]})
            hid = H.to(dev).requires_grad_(True)
            reps = head(hid, mask.to(dev))
            reps.backward(g[:, sh.start:sh.stop].to(dev))
            torch.cuda.synchronize(dev)
            assert head.weight.grad.shape == (sh.size, D)
            torch.save({"reps": reps.detach().cpu(), "dH": hid.grad.cpu(),
                        "dW": head.weight.grad.cpu(), "db": head.bias.grad.cpu(),
                        "shard": (sh.start, sh.stop)},
                       os.path.join(out_dir, f"r{rank}_{tag}.pt"))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("reduce", ["peer", "nccl"])
@pytest.mark.parametrize("world", [2, 4])
def test_sharded_head_matches_single_gpu(tmp_path, world, reduce):
    from sparton_b200.head import SpartonHead

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), reduce), nprocs=world,
                       join=True, start_method="spawn")
    H, W, b, mask, g = synthetic(B, S, D, V, (20, S), dtype=torch.bfloat16, seed=5, w_std=0.06)
    dev = torch.device("cuda", 0)
    head = SpartonHead(V, D, use_bias=True).to(dev, torch.bfloat16)
    head.load({"weight": W, "bias": b})
    hid = H.to(dev).requires_grad_(True)
    reps = head(hid, mask.to(dev))
    reps.backward(g.to(dev))
    ref = {"reps": reps.detach().cpu(), "dH": hid.grad.cpu(), "dW": head.weight.grad.cpu(),
           "db": head.bias.grad.cpu()}
    for tag in ("one", "rows", "tied"):
        covered = 0
        for r in range(world):
            got = torch.load(tmp_path / f"r{r}_{tag}.pt")
            lo, hi = got["shard"]
            covered += hi - lo
            assert torch.equal(got["reps"], ref["reps"][:, lo:hi]), (tag, r, "reps")
            assert torch.equal(got["dW"], ref["dW"][lo:hi]), (tag, r, "dW")
            assert torch.equal(got["db"], ref["db"][lo:hi]), (tag, r, "db")
            a, e = got["dH"].double(), ref["dH"].double()
            tol = 1e-2 * e.abs() + 1e-2 * e.abs().max()
            assert ((a - e).abs() <= tol).all(), (tag, r, float((a - e).abs().max()))
        assert covered == V
