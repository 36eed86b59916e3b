"""GPU parity of the training losses (sparton_b200.losses): the fused
regulariser kernels (csrc/reg.cu, through the C ABI) and the InfoNCE scoring,
against the loss oracle (oracle/losses_oracle.py, pinned to the reference's own
training functions).

Criteria: regulariser values within rtol 1e-5 (fp32 accumulation of B*V terms)
of the fp64 oracle on the same (dtype-rounded) inputs; their gradients within
one rounding of the output dtype (rtol 1e-2 for bf16 / f16, 1e-5 for fp32) plus
an absolute allowance of that rtol times the largest entry; InfoNCE loss and
gradients within rtol 1e-4 (fp32 scores) / the dtype's rounding."""
import numpy as np
import pytest
import torch

from oracle import losses_oracle as lo
from sparton_b200 import _lib, losses

pytestmark = pytest.mark.gpu

RTOL = {torch.bfloat16: 1e-2, torch.float16: 1e-2, torch.float32: 1e-5}
SHAPES = [(1, 1), (4, 257), (128, 30522), (7, 100)]


def _reps(B, V, dtype, seed, signed=False):
    gen = torch.Generator().manual_seed(seed)
    x = torch.rand(B, V, generator=gen) * 3.0
    x[torch.rand(B, V, generator=gen) < 0.5] = 0.0
    if signed:
        x = x - 1.0
    return x.to(dtype)


def _close(ours, ref, rtol, what):
    ours = ours.detach().double().cpu().numpy()
    np.testing.assert_allclose(ours, ref, rtol=rtol, atol=rtol * max(np.abs(ref).max(), 1e-30),
                               err_msg=what)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "B{}V{}".format(*s))
def test_regularizers_match_oracle(dtype, shape):
    B, V = shape
    x = _reps(B, V, dtype, seed=B + V, signed=(dtype == torch.float32)).cuda().requires_grad_(True)
    l1, fl = losses.regularizers(x)
    (0.7 * l1 + 1.3 * fl).backward()
    xn = x.detach().double().cpu().numpy()
    want_l1, g1 = lo.l1(xn)
    want_fl, gf = lo.flops(xn)
    np.testing.assert_allclose(l1.item(), want_l1, rtol=1e-5)
    np.testing.assert_allclose(fl.item(), want_fl, rtol=1e-5)
    _close(x.grad, 0.7 * g1 + 1.3 * gf, RTOL[dtype], "d(0.7*l1 + 1.3*flops)/dreps")


def test_regularizer_functions_and_determinism():
    x = _reps(64, 5000, torch.bfloat16, seed=9).cuda()
    a = losses.regularizers(x)
    b = losses.regularizers(x)
    assert a[0].item() == b[0].item() and a[1].item() == b[1].item()
    assert losses.l1_regularization(x).item() == a[0].item()
    assert losses.flops_regularization(x).item() == a[1].item()


def test_reg_capi_direct():
    """sparton_reg_fwd / sparton_reg_bwd through the C ABI, as a host binding calls them."""
    lib = _lib.load()
    x = _reps(16, 999, torch.bfloat16, seed=4).cuda()
    colsum = torch.empty(999, dtype=torch.float32, device="cuda")
    out = torch.empty(2, dtype=torch.float32, device="cuda")
    ws = torch.zeros(lib.sparton_reg_workspace_size(16, 999), dtype=torch.uint8, device="cuda")
    sh = torch.cuda.current_stream().cuda_stream
    assert lib.sparton_reg_fwd(x.data_ptr(), 2, 16, 999, 0.5, 0.25, colsum.data_ptr(),
                               out.data_ptr(), ws.data_ptr(), ws.numel(), sh) == 0
    g1 = torch.tensor([3.0], device="cuda")
    grad = torch.empty_like(x)
    assert lib.sparton_reg_bwd(x.data_ptr(), colsum.data_ptr(), g1.data_ptr(), None, 0.5, 0.25,
                               2, 16, 999, grad.data_ptr(), sh) == 0
    torch.cuda.synchronize()
    xn = x.double().cpu().numpy()
    np.testing.assert_allclose(colsum.cpu().numpy(), xn.sum(0), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(out.cpu().numpy(),
                               [0.5 * np.abs(xn).sum(), 0.25 * (xn.sum(0) ** 2).sum()], rtol=1e-5)
    _close(grad, 1.5 * np.sign(xn), 1e-2, "grad (g_flops NULL counts as 0)")
    # a workspace that is too small is refused before anything is launched
    assert lib.sparton_reg_fwd(x.data_ptr(), 2, 16, 999, 0.5, 0.25, colsum.data_ptr(),
                               out.data_ptr(), ws.data_ptr(), 8, sh) == 3


@pytest.mark.parametrize("shape", [(32, 32, 3000, 0.05), (21, 30, 2999, 0.05),
                                   (128, 128, 30522, 100.0)],
                         ids=lambda s: "Bq{}Bd{}V{}".format(*s[:3]))
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_info_nce_matches_oracle(dtype, shape):
    """16-bit reps run on the tensor-core GEMM (zero-padded to 16-byte rows:
    batch sizes not multiples of 8, an odd vocabulary); fp32 on torch. The
    full-vocabulary case uses a temperature that keeps the logits O(1): its
    scores (~1.7e4 from 30522 dense terms) carry fp32 rounding of ~1e-3, which
    at temperature 0.05 alone would move the softmax gradients by more than
    the tolerance."""
    Bq, Bd, V, temp = shape
    q = _reps(Bq, V, dtype, seed=1).cuda().requires_grad_(True)
    d = _reps(Bd, V, dtype, seed=2).cuda().requires_grad_(True)
    loss = losses.info_nce_loss(q, d, temperature=temp)
    loss.backward()
    want, dq, dd = lo.info_nce(q.detach().double().cpu().numpy(), d.detach().double().cpu().numpy(),
                               temp)
    np.testing.assert_allclose(loss.item(), want, rtol=1e-4)
    r = max(RTOL[dtype], 1e-4)
    _close(q.grad, dq, r, "dq")
    _close(d.grad, dd, r, "dd")


def test_info_nce_rejects_more_queries_than_documents():
    q = _reps(30, 64, torch.bfloat16, seed=1).cuda()
    d = _reps(21, 64, torch.bfloat16, seed=2).cuda()
    with pytest.raises(ValueError):
        losses.info_nce_loss(q, d)


def test_losses_reject_cpu_tensors():
    with pytest.raises(ValueError):
        losses.regularizers(torch.rand(2, 3))
