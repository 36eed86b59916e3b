"""GPU parity of the forward (the fused tcgen05 kernel for bf16 / f16, the FMA
kernel for fp32) against the CPU oracle, through the C ABI.

Criteria (written here, used by every test):
* reps: |ours - oracle| <= rtol*|oracle| + atol, rtol = 1e-2 for bf16/f16
  (outputs are stored in 16 bits) and 1e-5 for fp32, atol = 1e-3 / 1e-5;
* idx: bit-exact equal to the oracle's first-argmax, except at near-ties
  (top-2 valid logits, or the max and 0, within 2^-16 * sum|h*w| — the fp32
  accumulation error bound), where any candidate within that bound is accepted.
"""
import ctypes

import numpy as np
import pytest
import torch

import sparton_b200.ops  # noqa: F401  (registers torch.ops.sparton.*)
from oracle import sparton_oracle as orc
from sparton_b200 import _lib
from tests._cases import DTYPES, golden_names, load_golden, np64, synthetic

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: (1e-2, 1e-3), torch.float16: (1e-2, 1e-3), torch.float32: (1e-5, 1e-5)}


def run_fwd(H, W, b, mask):
    dev = torch.device("cuda")
    reps, idx = torch.ops.sparton.fused_sparton_fwd(
        H.to(dev), W.to(dev), None if b is None else b.to(dev), mask.to(dev))
    torch.cuda.synchronize()
    return reps.cpu(), idx.cpu()


def check_fwd(H, W, b, mask, reps, idx):
    rtol, atol = TOL[H.dtype]
    mask_np = (mask != 0).numpy().astype(np.int64)
    ref, ref_idx, _ = orc.forward(np64(H), np64(W), np64(b), mask_np)
    np.testing.assert_allclose(np64(reps), ref, rtol=rtol, atol=atol)
    ok = orc.accept_indices(idx.numpy(), np64(H), np64(W), np64(b), mask_np)
    bad = np.argwhere(~ok)
    assert ok.all(), f"{len(bad)} argmax mismatches outside near-ties, first {bad[:5].tolist()}"
    exact = (idx.numpy() == ref_idx).mean()
    assert exact > 0.99, f"only {exact:.4f} of indices equal the oracle's"


SHAPES = [
    # B, S, D, V, lengths, bias
    (1, 1, 64, 1, (1, 1), True),
    (3, 70, 64, 300, (1, 70), True),
    (2, 600, 128, 257, (300, 600), True),     # several s-tiles per row
    (4, 33, 72, 130, (0, 33), False),          # D not a multiple of 64, empty rows
    (4, 256, 768, 1000, (32, 256), True),      # config-2 row shape
    (2, 128, 4096, 300, (64, 128), False),     # config-5 hidden size
    (300, 8, 64, 200, (1, 8), True),           # many short rows: scheduler
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "B{}S{}D{}V{}".format(*s[:4]))
def test_fwd_tensor_core_matches_oracle(dtype, shape):
    B, S, D, V, lengths, bias = shape
    H, W, b, mask, _ = synthetic(B, S, D, V, lengths, dtype=dtype, use_bias=bias,
                                 w_std=0.5 / D ** 0.5, seed=B * 7 + S)
    reps, idx = run_fwd(H, W, b, mask)
    assert reps.dtype == dtype and idx.dtype == torch.int32
    check_fwd(H, W, b, mask, reps, idx)


@pytest.mark.parametrize("shape", SHAPES[:5], ids=lambda s: "B{}S{}D{}V{}".format(*s[:4]))
def test_fwd_fp32_matches_oracle(shape):
    B, S, D, V, lengths, bias = shape
    H, W, b, mask, _ = synthetic(B, S, D, V, lengths, dtype=torch.float32, use_bias=bias,
                                 w_std=0.5 / D ** 0.5, seed=B + S)
    reps, idx = run_fwd(H, W, b, mask)
    check_fwd(H, W, b, mask, reps, idx)


@pytest.mark.parametrize("mask_dtype", [torch.bool, torch.int32, torch.int64, torch.float32,
                                        torch.uint8, torch.bfloat16])
def test_mask_dtypes_and_holes(mask_dtype):
    H, W, b, mask, _ = synthetic(3, 90, 128, 333, (10, 90), dtype=torch.bfloat16, seed=11,
                                 w_std=0.05, holes=True)
    reps, idx = run_fwd(H, W, b, mask.to(mask_dtype))
    check_fwd(H, W, b, mask, reps, idx)


def test_all_rows_empty():
    H, W, b, mask, _ = synthetic(2, 40, 64, 150, (0, 0), dtype=torch.bfloat16, seed=3)
    reps, idx = run_fwd(H, W, b, mask)
    assert (reps == 0).all() and (idx == 0).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rows_do_not_leak_into_each_other(dtype):
    """The tensor-core forward lays the positions of consecutive rows end to end
    and cuts that stream into tiles and work units. Rows here alternate between
    hidden states of size ~1 and ~30 and have lengths of 16 mod 32 (a row or a
    unit then ends in the middle of a 32-column chunk), so a position of the
    next row counted into a row's max would show as a large error."""
    B, S, D, V = 40, 200, 64, 300
    gen = torch.Generator().manual_seed(11)
    H = torch.randn(B, S, D, generator=gen)
    H[1::2] *= 30.0
    W = torch.randn(V, D, generator=gen) * (0.5 / D ** 0.5)
    b = torch.randn(V, generator=gen) * 0.05
    lengths = torch.tensor([16 + 32 * (i % 6) for i in range(B)])
    lengths[5] = 0
    lengths[17] = 0
    mask = (torch.arange(S)[None, :] < lengths[:, None]).to(torch.int64)
    H, W, b = H.to(dtype), W.to(dtype), b.to(dtype)
    reps, idx = run_fwd(H, W, b, mask)
    check_fwd(H, W, b, mask, reps, idx)


@pytest.mark.parametrize("name", golden_names())
def test_golden_fixtures_on_gpu(name):
    """Same inputs as the reference run that produced the fixture; fp64
    fixtures are fed in fp32."""
    c = load_golden(name)
    dt = DTYPES[c["dtype"]]
    dt = torch.float32 if dt == torch.float64 else dt
    H = torch.tensor(c["H"]).to(dt)
    W = torch.tensor(c["W"]).to(dt)
    b = torch.tensor(c["bias"]).to(dt) if c["has_bias"] else None
    mask = torch.tensor(c["mask"])
    reps, idx = run_fwd(H, W, b, mask)
    rtol, atol = TOL[dt]
    np.testing.assert_allclose(np64(reps), c["reps"], rtol=rtol, atol=atol)
    check_fwd(H, W, b, mask, reps, idx)


def test_full_size_config2_sampled_columns():
    """B=128 S=256 D=768 V=30522 bf16, lengths U[32,256]: every output checked for
    the size-independent properties, 160 vocab columns (incl. the ragged last
    tile) against the oracle."""
    B, S, D, V = 128, 256, 768, 30522
    H, W, b, mask, _ = synthetic(B, S, D, V, (32, 256), dtype=torch.bfloat16, seed=0)
    reps, idx = run_fwd(H, W, b, mask)
    reps2, idx2 = run_fwd(H, W, b, mask)
    assert torch.equal(reps, reps2) and torch.equal(idx, idx2), "not deterministic"
    L = mask.sum(1)
    assert (reps >= 0).all()
    assert (idx >= 0).all() and (idx < L[:, None].clamp(min=1)).all()
    assert ((reps == 0) <= (idx == 0)).all()
    rng = np.random.default_rng(0)
    sel = np.unique(np.concatenate([rng.choice(V, 140, replace=False), np.arange(V - 20, V)]))
    sel_t = torch.tensor(sel)
    check_fwd(H, W[sel_t], b[sel_t], mask, reps[:, sel_t], idx[:, sel_t])


def test_capi_direct_and_device_status():
    """Drives sparton_mask_prepare + sparton_fwd_prepared through ctypes with
    torch-allocated buffers; the device status word stays 0."""
    lib = _lib.load()
    B, S, D, V = 5, 77, 256, 700
    H, W, b, mask, _ = synthetic(B, S, D, V, (1, 77), dtype=torch.bfloat16, seed=5, w_std=0.03)
    dev = torch.device("cuda")
    H, W, b, mask = H.to(dev), W.to(dev), b.to(dev), mask.to(dev)
    reps = torch.empty(B, V, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(B, V, dtype=torch.int32, device=dev)
    ws = torch.empty(lib.sparton_fwd_workspace_size(B, S, D, V), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.sparton_mask_prepare(mask.data_ptr(), 2, B, S, ws.data_ptr(), ws.numel(), stream) == 0
    assert lib.sparton_fwd_prepared(H.data_ptr(), W.data_ptr(), b.data_ptr(), 2, B, S, D, V,
                                    reps.data_ptr(), idx.data_ptr(), ws.data_ptr(), ws.numel(),
                                    stream) == 0
    assert _lib.read_device_status(ws) == 0
    check_fwd(H.cpu(), W.cpu(), b.cpu(), mask.cpu(), reps.cpu(), idx.cpu())


def test_rejects_cpu_tensors_and_bad_shapes():
    H, W, b, mask, _ = synthetic(2, 8, 64, 10, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        torch.ops.sparton.fused_sparton_fwd(H, W, b, mask)
    with pytest.raises(ValueError):
        torch.ops.sparton.fused_sparton_fwd(H.cuda(), W[:, :32].cuda(), b.cuda(), mask.cuda())
    with pytest.raises(ValueError):
        torch.ops.sparton.fused_sparton_fwd(H.cuda(), W.float().cuda(), b.cuda(), mask.cuda())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_inference_forward_without_idx(dtype):
    """The inference forward (idx NULL through the C ABI, the
    fused_sparton_fwd_scores op) writes the same reps as the training forward,
    bit for bit, and SpartonHead takes it when autograd is off."""
    from sparton_b200.head import SpartonHead

    B, S, D, V = 9, 300, 256, 1100
    H, W, b, mask, _ = synthetic(B, S, D, V, (0, 300), dtype=dtype, seed=41, w_std=0.03)
    dev = torch.device("cuda")
    Hd, Wd, bd, md = H.to(dev), W.to(dev), b.to(dev), mask.to(dev)
    reps, idx = torch.ops.sparton.fused_sparton_fwd(Hd, Wd, bd, md)
    scores = torch.ops.sparton.fused_sparton_fwd_scores(Hd, Wd, bd, md)
    torch.cuda.synchronize()
    assert torch.equal(scores.cpu(), reps.cpu())
    head = SpartonHead(V, D, use_bias=True).to(dev, dtype)
    head.load({"weight": Wd, "bias": bd})
    with torch.no_grad():
        r_nograd = head(Hd, md)
    with torch.inference_mode():
        r_inf = head(Hd, md)
    assert not r_nograd.requires_grad
    assert torch.equal(r_nograd.cpu(), reps.cpu()) and torch.equal(r_inf.cpu(), reps.cpu())
    check_fwd(H, W, b, mask, scores.cpu(), idx.cpu())
