"""Failure detection without faulting, trapping or hanging a GPU.

* GPU: a device wait that nobody completes gives up after its limit, records a
  status code the host reads, and leaves the context usable
  (``sparton_selftest_wait_timeout`` waits through the same bounded-wait
  routine as the forward kernel, with a short limit).
* CPU, 2 gloo ranks: a rank that stops taking part between steps (it stalls,
  or its process exits) makes its peer's next collective of the sharded
  backward (``_HiddenGradReducer``: the all-reduce of the partial d_hidden)
  end with an error within the process group's timeout, instead of hanging.
  The native operators are replaced by CPU stand-ins (as in
  test_sharding_gloo), so only host logic and collectives run.
"""
import ctypes
import datetime
import multiprocessing
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist

from sparton_b200 import _lib


# --------------------------------------------------------------------- GPU
@pytest.mark.gpu
@pytest.mark.parametrize("limit_us", [1000, 20000])
def test_device_wait_times_out_with_a_status(limit_us):
    lib = _lib.load()
    dev = torch.device("cuda")
    ws = torch.zeros(256, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(lib.sparton_selftest_wait_timeout(limit_us, ws.data_ptr(), ws.numel(), stream),
               "sparton_selftest_wait_timeout")
    assert _lib.read_device_status(ws) == 0x1F0  # SPARTON_DEV_TIMEOUT_SELFTEST
    words = ws.view(torch.int32).cpu().numpy()
    waited_us, left_on_abort = int(words[1]), int(words[2])
    assert limit_us <= waited_us < limit_us + 500000, waited_us
    assert left_on_abort == 1
    # The context is intact: a forward right after it runs and reports status 0.
    import sparton_b200.ops  # noqa: F401
    from tests._cases import synthetic

    H, W, b, mask, _ = synthetic(2, 40, 64, 200, (1, 40), dtype=torch.bfloat16, seed=2)
    fws = torch.empty(lib.sparton_fwd_workspace_size(2, 40, 64, 200), dtype=torch.uint8,
                      device=dev)
    reps = torch.empty(2, 200, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(2, 200, dtype=torch.int32, device=dev)
    Hd, Wd, bd, md = H.to(dev), W.to(dev), b.to(dev), mask.to(dev)
    _lib.check(lib.sparton_fwd(Hd.data_ptr(), Wd.data_ptr(), bd.data_ptr(), md.data_ptr(), 2, 2,
                               2, 40, 64, 200, reps.data_ptr(), idx.data_ptr(), fws.data_ptr(),
                               fws.numel(), stream), "sparton_fwd")
    assert _lib.read_device_status(fws) == 0
    ref, _ = torch.ops.sparton.fused_sparton_fwd(Hd, Wd, bd, md)
    assert torch.equal(ref, reps)


def test_selftest_rejects_bad_arguments():
    lib = _lib.load()
    assert lib.sparton_selftest_wait_timeout(0, None, 0, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.sparton_selftest_wait_timeout(2000000, None, 0, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.sparton_selftest_wait_timeout(10, None, 0, None) == _lib.ERR_WORKSPACE
    assert (lib.sparton_selftest_wait_timeout(10, ctypes.c_void_p(0x1001), 256, None)
            == _lib.ERR_INVALID_ARGUMENT)


# --------------------------------------------------------------------- gloo
PG_TIMEOUT_S = 3.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sharded_step(head, H, mask, g):
    sh = head.shard
    hid = H.clone().requires_grad_(True)
    head(hid, mask).backward(g[:, sh.start:sh.stop])
    return hid.grad


def _rank(rank, world, port, mode, results):
    """Both ranks run one sharded step; then rank 1 leaves (stalls or exits)
    and rank 0 runs a second step, whose d_hidden all-reduce must fail."""
    from sparton_b200 import ops
    from sparton_b200.head import SpartonHead
    from tests import test_sharding_gloo as sg

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    ops.forward_impl = sg._cpu_forward
    ops.backward_impl = sg._cpu_backward
    ops.hidden_grad_rows = sg._cpu_hidden_rows
    H, W, b, mask, g = sg._inputs()
    head = SpartonHead(sg.V, sg.D, use_bias=True, process_group=dist.group.WORLD).double()
    head.load({"weight": W, "bias": b})
    _sharded_step(head, H, mask, g)  # step 1: every rank takes part
    if rank == 1:
        if mode == "stall":
            time.sleep(4 * PG_TIMEOUT_S)  # between steps, nothing in flight
        os._exit(0)  # leaves without destroying the group
    t0 = time.monotonic()
    try:
        _sharded_step(head, H, mask, g)  # step 2: the peer is gone
        results.put(("no error", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        results.put((type(e).__name__ + ": " + str(e)[:200], time.monotonic() - t0))
    os._exit(0)


@pytest.mark.timeout(120)
@pytest.mark.parametrize("mode", ["stall", "exit"])
def test_peer_that_leaves_between_steps_ends_the_collective_with_an_error(mode):
    ctx = multiprocessing.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, mode, results)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        outcome, waited = results.get(timeout=90)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():  # our own child only
                p.kill()
                p.join()
    assert outcome != "no error", "the collective succeeded without its peer"
    # An exited peer is noticed at once (connection closed); a stalled one when
    # the process group's timeout expires. Either way well before a hang.
    assert waited < 10 * PG_TIMEOUT_S, (outcome, waited)
    print(f"{mode}: rank 0 got '{outcome}' after {waited:.2f} s")
