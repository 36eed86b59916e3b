"""GPU parity of the MLM transform (csrc/transform.cu through the C ABI and
sparton_b200.transform) with the oracle (oracle/transform_oracle.py, pinned to
the reference's own ProjectionPyTorch on BERT / RoBERTa transforms).

Criteria: the gelu + LayerNorm kernels against the oracle on the same y, with
the gelu output rounded to the input dtype as the reference's modules do:
h within rtol 1e-2 (16-bit; one rounding of h plus the rounded gelu output
scaled by rstd) / 1e-5 (fp32), plus the same fraction of max|h|; dy, d_gamma,
d_beta, d_bias within 2e-2 / 1e-4 of the oracle relative to the largest entry.
The whole projection in fp32 against the reference fixtures: reps and
gradients within 1e-4 of the largest entry (fp32 GEMMs and sums against the
reference's float64 run)."""
import glob
import os

import numpy as np
import pytest
import torch
from torch import nn

from oracle import transform_oracle as to
from sparton_b200 import transform as tr

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURES = sorted(os.path.basename(p)[:-4]
                  for p in glob.glob(os.path.join(HERE, "golden", "transform_*.npz")))
NAME = {torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32"}
TOL = {torch.bfloat16: 1e-2, torch.float16: 1e-2, torch.float32: 1e-5}


def close(ours, ref, tol, what):
    ours = ours.detach().double().cpu().numpy()
    ref = np.asarray(ref)
    np.testing.assert_allclose(ours, ref, rtol=tol, atol=tol * max(np.abs(ref).max(), 1e-30),
                               err_msg=what)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 32), (7, 100), (300, 768), (40, 1024), (9, 4096)],
                         ids=lambda s: "rows{}D{}".format(*s))
def test_gelu_layernorm_kernels(dtype, shape):
    rows, D = shape
    gen = torch.Generator().manual_seed(rows + D)
    y = (torch.randn(rows, D, generator=gen) * 1.5).to(dtype)
    gamma = (1 + 0.2 * torch.randn(D, generator=gen)).to(dtype)
    beta = (0.1 * torch.randn(D, generator=gen)).to(dtype)
    dh = torch.randn(rows, D, generator=gen).to(dtype)
    eps = 1e-12 if D == 768 else 1e-5
    h, mean, rstd = tr.transform_fwd_impl(y.cuda(), gamma.cuda(), beta.cuda(), eps)
    ref_h, cache = to.layer_norm_gelu(y.double().numpy(), gamma.double().numpy(),
                                      beta.double().numpy(), eps, NAME[dtype])
    close(h, ref_h, TOL[dtype], "h")
    np.testing.assert_allclose(rstd.cpu().numpy(), cache[4][:, 0], rtol=1e-4)
    dy, dg, db, dbias = tr.transform_bwd_impl(dh.cuda(), y.cuda(), gamma.cuda(), mean, rstd)
    rdy, rdg, rdb = to.layer_norm_gelu_backward(dh.double().numpy(), cache)
    t = 2e-2 if dtype != torch.float32 else 1e-4
    close(dy, rdy, t, "dy")
    close(dg, rdg, t, "d_gamma")
    close(db, rdb, t, "d_beta")
    close(dbias, rdy.sum(axis=0), t, "d_bias")


def test_kernels_deterministic_and_no_param_grads():
    gen = torch.Generator().manual_seed(3)
    y = torch.randn(1000, 768, generator=gen).to(torch.bfloat16).cuda()
    gamma = torch.ones(768, dtype=torch.bfloat16, device="cuda")
    beta = torch.zeros(768, dtype=torch.bfloat16, device="cuda")
    dh = torch.randn(1000, 768, generator=gen).to(torch.bfloat16).cuda()
    h1, m1, r1 = tr.transform_fwd_impl(y, gamma, beta, 1e-5)
    h2, m2, r2 = tr.transform_fwd_impl(y, gamma, beta, 1e-5)
    assert torch.equal(h1, h2)
    a = tr.transform_bwd_impl(dh, y, gamma, m1, r1)
    b = tr.transform_bwd_impl(dh, y, gamma, m1, r1)
    for x, z in zip(a, b):
        assert torch.equal(x, z)
    dy, dg, db, dbias = tr.transform_bwd_impl(dh, y, gamma, m1, r1, need_params=False)
    assert torch.equal(dy, a[0]) and dg is None and db is None and dbias is None


@pytest.mark.parametrize("name", FIXTURES)
def test_projection_matches_reference_fixture(name):
    """SpartonProjection in fp32 against the reference's ProjectionPyTorch (float64)."""
    c = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    dev = torch.device("cuda")
    D, V = c["W"].shape[1], c["W"].shape[0]
    dense = nn.Linear(D, D).to(dev)
    ln = nn.LayerNorm(D, eps=float(c["eps"])).to(dev)
    decoder = nn.Linear(D, V).to(dev)
    with torch.no_grad():
        for mod, w, b in ((dense, "Wd", "bd"), (ln, "gamma", "beta"), (decoder, "W", "b")):
            mod.weight.copy_(torch.tensor(c[w]))
            mod.bias.copy_(torch.tensor(c[b]))

    class RobertaLike(nn.Module):  # the reference's RobertaTransform layout
        def __init__(self):
            super().__init__()
            self.dense, self.layer_norm = dense, ln

    proj = tr.SpartonProjection(RobertaLike(), decoder)
    x = torch.tensor(c["x"], dtype=torch.float32, device=dev).requires_grad_(True)
    reps = proj(x, torch.tensor(c["mask"], device=dev))
    reps.backward(torch.tensor(c["g"], dtype=torch.float32, device=dev))
    t = 1e-4
    close(reps, c["reps"], t, "reps")
    close(x.grad, c["dx"], t, "dx")
    close(dense.weight.grad, c["dWd"], t, "dWd")
    close(dense.bias.grad, c["dbd"], t, "dbd")
    close(ln.weight.grad, c["dgamma"], t, "dgamma")
    close(ln.bias.grad, c["dbeta"], t, "dbeta")
    close(decoder.weight.grad, c["dW"], t, "dW")
    close(decoder.bias.grad, c["db"], t, "db")


def test_projection_from_bert_transform_bf16():
    """SpartonProjection built from transformers' BERT predictions.transform
    (bf16), against the oracle projection on the same bf16 parameters."""
    transformers = pytest.importorskip("transformers")
    cfg = transformers.BertConfig(vocab_size=500, hidden_size=64, num_hidden_layers=1,
                                  num_attention_heads=2, intermediate_size=128)
    torch.manual_seed(0)
    llm = transformers.BertForMaskedLM(cfg).cuda().to(torch.bfloat16)
    transform, decoder = llm.cls.predictions.transform, llm.cls.predictions.decoder
    proj = tr.SpartonProjection(transform, decoder)
    assert proj.sparton_head.weight is decoder.weight  # tied
    gen = torch.Generator().manual_seed(1)
    B, S = 4, 40
    x = torch.randn(B, S, 64, generator=gen).to(torch.bfloat16).cuda()
    mask = (torch.arange(S)[None, :] < torch.tensor([40, 17, 3, 29])[:, None]).to(torch.int64)
    with torch.no_grad():
        reps = proj(x, mask.cuda())
    p = lambda t: t.detach().double().cpu().numpy()  # noqa: E731
    ref_h, _ = to.transform_forward(p(x), p(transform.dense.weight), p(transform.dense.bias),
                                    p(transform.LayerNorm.weight), p(transform.LayerNorm.bias),
                                    transform.LayerNorm.eps, "bfloat16")
    from oracle import sparton_oracle as orc
    ref_reps, _, _ = orc.forward(ref_h, p(decoder.weight), p(decoder.bias), mask.numpy())
    # the reference rounds y and h to bf16 as well; the head sums over D = 64 products
    close(reps, ref_reps, 3e-2, "reps")


def test_rejects_approximate_gelu():
    class T(nn.Module):
        def __init__(self):
            super().__init__()
            self.dense = nn.Linear(8, 8)
            self.transform_act_fn = nn.GELU(approximate="tanh")
            self.LayerNorm = nn.LayerNorm(8)

    with pytest.raises(ValueError):
        tr.MLMTransform.from_module(T())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_dense_layer_on_the_tensor_core_gemm(dtype):
    """The dense layer of the transform and its two backward products run on
    sparton_gemm for 16-bit inputs: y = x W^T + b, dx = dy W, dW = dy^T x,
    against torch fp32 products of the same 16-bit values (one rounding of the
    output dtype plus 1e-3 of the sum of |terms|)."""
    B, S, D_in, D_out = 3, 77, 256, 192
    gen = torch.Generator().manual_seed(8)
    x = torch.randn(B, S, D_in, generator=gen).to(dtype).cuda()
    w = (torch.randn(D_out, D_in, generator=gen) * 0.05).to(dtype).cuda()
    b = (torch.randn(D_out, generator=gen) * 0.1).to(dtype).cuda()
    dy = torch.randn(B, S, D_out, generator=gen).to(dtype).cuda()
    assert tr._tensor_core(x, w)
    y = tr._dense_fwd(x, w, b)
    dx, dw = tr._dense_bwd(dy, x, w, True, True)
    torch.cuda.synchronize()
    xf, wf, dyf = x.float().reshape(-1, D_in), w.float(), dy.float().reshape(-1, D_out)
    rt = 2 ** -8 if dtype == torch.bfloat16 else 2 ** -11
    for name, ours, ref, mag in (
            ("y", y.reshape(-1, D_out), xf @ wf.t() + b.float(), xf.abs() @ wf.abs().t()),
            ("dx", dx.reshape(-1, D_in), dyf @ wf, dyf.abs() @ wf.abs()),
            ("dW", dw, dyf.t() @ xf, dyf.abs().t() @ xf.abs())):
        assert ours.dtype == dtype
        err = (ours.float() - ref).abs()
        bad = err > rt * ref.abs() + 1e-3 * mag + 1e-6
        assert not bad.any(), (name, int(bad.sum()), float(err.max()))


def test_projection_bf16_backward_matches_torch_transform():
    """SpartonProjection (bf16) forward + backward against the same head behind
    the transform as torch modules (nn.Linear on cuBLAS, gelu, nn.LayerNorm):
    the gradients of every parameter and of the input agree within bf16
    rounding of sums (rtol 3e-2 plus 3e-2 of the largest entry) on at least
    99% of their elements. Not all: the two paths round the hidden states
    differently, so an argmax at a near-tie may pick another position, which
    moves that (b, v) pair's gradient to another row."""
    from torch import nn

    B, S, D, V = 4, 64, 128, 700
    gen = torch.Generator().manual_seed(21)
    dense = nn.Linear(D, D).cuda().to(torch.bfloat16)
    ln = nn.LayerNorm(D, eps=1e-12).cuda().to(torch.bfloat16)
    decoder = nn.Linear(D, V).cuda().to(torch.bfloat16)

    class T(nn.Module):
        def __init__(self):
            super().__init__()
            self.dense, self.layer_norm = dense, ln

        def forward(self, t):
            return self.layer_norm(torch.nn.functional.gelu(self.dense(t)))

    t = T()
    proj = tr.SpartonProjection(t, decoder)
    x = torch.randn(B, S, D, generator=gen).to(torch.bfloat16).cuda()
    mask = (torch.arange(S)[None, :] < torch.tensor([64, 30, 9, 50])[:, None]).cuda()
    g = torch.randn(B, V, generator=gen).to(torch.bfloat16).cuda()
    params = [dense.weight, dense.bias, ln.weight, ln.bias, decoder.weight, decoder.bias]

    def grads(fn):
        for p_ in params:
            p_.grad = None
        xi = x.detach().requires_grad_(True)
        fn(xi).backward(g)
        return [xi.grad.float()] + [p_.grad.float() for p_ in params]

    ours = grads(lambda xi: proj(xi, mask))
    ref = grads(lambda xi: proj.sparton_head(t(xi), mask))
    for i, (a, e) in enumerate(zip(ours, ref)):
        tol = 3e-2 * e.abs() + 3e-2 * e.abs().max()
        frac = float(((a - e).abs() <= tol).float().mean())
        assert frac >= 0.99, (i, frac, float((a - e).abs().max()))
