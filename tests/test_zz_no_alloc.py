"""sparton_fwd_noalloc: the forward for callers that cannot allocate device memory.

Who needs it: a host that binds the C ABI from Go or Java (cgo / JNI) without a
CUDA allocator of its own, a process whose framework already reserved the
device memory for its own pool (so cudaMalloc would fail), or a loop that must
not call cudaMalloc because it can synchronise the device. Instead of a
caller-provided workspace, the entry point uses a fixed scratch array compiled
into the library, shared by every call on the device.

The test calls the entry point through the C ABI twice in a row, with
different shapes and masks, and checks each result against sparton_fwd (the
entry point with a caller workspace). Both run the same kernels on the same
inputs, so reps and idx must be bit-identical (torch.equal), and the device
status word that sparton_fwd_noalloc_status reads back must be 0 after each
call. The second call reuses the scratch left by the first, so it also shows
that nothing stale leaks between calls. This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

from sparton_b200 import _lib
from tests._cases import synthetic

pytestmark = pytest.mark.gpu


def _with_workspace(lib, H, W, b, mask):
    B, S, D = H.shape
    V = W.shape[0]
    reps = torch.empty(B, V, dtype=H.dtype, device=H.device)
    idx = torch.empty(B, V, dtype=torch.int32, device=H.device)
    ws = torch.empty(lib.sparton_fwd_workspace_size(B, S, D, V), dtype=torch.uint8, device=H.device)
    st = lib.sparton_fwd(H.data_ptr(), W.data_ptr(), b.data_ptr(), mask.data_ptr(),
                         _lib.MASK_DTYPE[mask.dtype], _lib.DTYPE[H.dtype], B, S, D, V,
                         reps.data_ptr(), idx.data_ptr(), ws.data_ptr(), ws.numel(),
                         torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "sparton_fwd")
    return reps, idx


def _without_workspace(lib, H, W, b, mask):
    B, S, D = H.shape
    V = W.shape[0]
    reps = torch.empty(B, V, dtype=H.dtype, device=H.device)
    idx = torch.empty(B, V, dtype=torch.int32, device=H.device)
    st = lib.sparton_fwd_noalloc(H.data_ptr(), W.data_ptr(), b.data_ptr(), mask.data_ptr(),
                                 _lib.MASK_DTYPE[mask.dtype], _lib.DTYPE[H.dtype], B, S, D, V,
                                 reps.data_ptr(), idx.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
    _lib.check(st, "sparton_fwd_noalloc")
    return reps, idx


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    lib = _lib.load()
    dev = torch.device("cuda")
    cases = [
        dict(B=6, S=200, D=256, V=1500, lengths=(1, 200), seed=1, holes=False),
        dict(B=3, S=70, D=128, V=700, lengths=(0, 70), seed=2, holes=True),
    ]
    for c in cases:
        H, W, b, mask, _ = synthetic(c["B"], c["S"], c["D"], c["V"], c["lengths"],
                                     dtype=torch.bfloat16, seed=c["seed"], w_std=0.04,
                                     holes=c["holes"])
        H, W, b, mask = H.to(dev), W.to(dev), b.to(dev), mask.to(dev)
        ref_reps, ref_idx = _with_workspace(lib, H, W, b, mask)
        reps, idx = _without_workspace(lib, H, W, b, mask)
        code = ctypes.c_uint32(0xFFFFFFFF)
        _lib.check(lib.sparton_fwd_noalloc_status(torch.cuda.current_stream().cuda_stream,
                                                  ctypes.byref(code)),
                   "sparton_fwd_noalloc_status")
        assert code.value == 0, f"device status {code.value:#x} after sparton_fwd_noalloc"
        torch.cuda.synchronize()
        assert torch.equal(reps.cpu(), ref_reps.cpu())
        assert torch.equal(idx.cpu(), ref_idx.cpu())


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    B, S, D, V = 4096, 8192, 64, 100  # needs ~4 MiB of scratch, the array holds 1 MiB
    assert lib.sparton_fwd_workspace_size(B, S, D, V) > (1 << 20)
    st = lib.sparton_fwd_noalloc(None, None, None, None, 2, 2, B, S, D, V, None, None, None)
    assert st == _lib.ERR_UNSUPPORTED
    assert "scratch" in _lib.last_error()
