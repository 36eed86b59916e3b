"""Pins the CPU oracle against fixtures produced by the reference's own torch
head (tests/golden/make_golden.py), before any GPU test relies on it."""
import numpy as np
import pytest
import torch

from oracle import sparton_oracle as orc
from oracle.torch_head import torch_head
from tests._cases import DTYPES, golden_names, load_golden

# Tolerances by the dtype the reference computed the fixture in: float64 is
# exact up to summation order; float32 up to fp32 rounding; 16-bit fixtures are
# computed in 16-bit arithmetic by the reference, so only reps are pinned there
# (rtol 1e-2, the bf16/fp16 parity bar).
RTOL = {"float64": 1e-10, "float32": 2e-5, "bfloat16": 1e-2, "float16": 1e-2}
ATOL = {"float64": 1e-12, "float32": 2e-6, "bfloat16": 1e-2, "float16": 2e-3}


def test_golden_fixtures_present():
    names = golden_names()
    assert len(names) >= 6, names


@pytest.mark.parametrize("name", golden_names())
def test_oracle_forward_matches_reference(name):
    c = load_golden(name)
    reps, idx, m = orc.forward(c["H"], c["W"], c["bias"], c["mask"])
    np.testing.assert_allclose(reps, c["reps"], rtol=RTOL[c["dtype"]], atol=ATOL[c["dtype"]])
    assert idx.dtype == np.int64 and (idx >= 0).all() and (idx < c["H"].shape[1]).all()


@pytest.mark.parametrize("name", [n for n in golden_names() if "f64" in n or "f32" in n])
def test_oracle_backward_matches_reference(name):
    c = load_golden(name)
    dH, dW, db = orc.backward_exact(c["g"], c["H"], c["W"], c["bias"], c["mask"])
    rt, at = RTOL[c["dtype"]], ATOL[c["dtype"]]
    np.testing.assert_allclose(dH, c["dH"], rtol=rt, atol=at)
    np.testing.assert_allclose(dW, c["dW"], rtol=rt, atol=at)
    if c["has_bias"]:
        np.testing.assert_allclose(db, c["db"], rtol=rt, atol=at)
    else:
        assert db is None


@pytest.mark.parametrize("name", [n for n in golden_names() if "f64" in n])
def test_kernel_formula_equals_torch_head_in_exact_arithmetic(name):
    # The fused kernel's g * exp(-score) (sparton_kernel.py:531) equals the torch
    # head's g / (1 + max) when score = log1p(max) is not rounded.
    c = load_golden(name)
    reps, idx, m = orc.forward(c["H"], c["W"], c["bias"], c["mask"])
    a = orc.backward_from_scores(c["g"], reps, idx, c["H"], c["W"], c["has_bias"])
    b = orc.backward_exact(c["g"], c["H"], c["W"], c["bias"], c["mask"])
    for x, y in zip(a, b):
        if x is None:
            assert y is None
        else:
            np.testing.assert_allclose(x, y, rtol=1e-12, atol=1e-14)


@pytest.mark.parametrize("name", golden_names())
def test_torch_head_restatement_matches_reference(name):
    c = load_golden(name)
    dt = DTYPES[c["dtype"]]
    H = torch.tensor(c["H"]).to(dt)
    W = torch.tensor(c["W"]).to(dt)
    b = torch.tensor(c["bias"]).to(dt) if c["has_bias"] else None
    reps = torch_head(H, W, b, torch.tensor(c["mask"]))
    np.testing.assert_allclose(reps.double().numpy(), c["reps"], rtol=1e-6, atol=1e-6)


def test_argmax_rule_first_index_and_zero_default():
    # Hand-built case: ties resolve to the smallest position, masked positions
    # never win, a non-positive max yields index 0 and value 0.
    H = np.zeros((1, 5, 2))
    H[0, 1] = [1.0, 0.0]
    H[0, 3] = [1.0, 0.0]   # tie with position 1 for vocab 0
    H[0, 4] = [5.0, 0.0]   # masked out
    H[0, 2] = [0.0, -1.0]
    W = np.array([[2.0, 0.0], [0.0, 1.0], [0.0, 0.0]])
    mask = np.array([[1, 1, 1, 1, 0]])
    reps, idx, m = orc.forward(H, W, None, mask)
    assert idx[0, 0] == 1 and np.isclose(reps[0, 0], np.log1p(2.0))
    assert idx[0, 1] == 0 and reps[0, 1] == 0.0   # max logit 0 -> (0, 0)
    assert idx[0, 2] == 0 and reps[0, 2] == 0.0


def test_near_tie_acceptance():
    H = np.zeros((1, 3, 1))
    H[0, :, 0] = [1.0, 1.0 + 1e-9, 0.5]
    W = np.ones((1, 1))
    mask = np.ones((1, 3))
    reps, idx, m = orc.forward(H, W, None, mask)
    assert idx[0, 0] == 1
    assert orc.near_tie_mask(H, W, None, mask)[0, 0]
    ok = orc.accept_indices(np.array([[0]]), H, W, None, mask)
    assert ok[0, 0]                                   # within tolerance of the max
    assert not orc.accept_indices(np.array([[2]]), H, W, None, mask)[0, 0]


def test_sharded_backward_sums_partials():
    rng = np.random.default_rng(0)
    B, S, D, V = 2, 9, 8, 40
    H = rng.standard_normal((B, S, D))
    W = rng.standard_normal((V, D)) * 0.3
    mask = np.ones((B, S))
    g = rng.standard_normal((B, V))
    reps, idx, _ = orc.forward(H, W, None, mask)
    full, _, _ = orc.backward_from_scores(g, reps, idx, H, W, False)
    cuts = [0, 13, 27, 40]
    parts = [slice(cuts[i], cuts[i + 1]) for i in range(3)]
    total = orc.sharded_backward_hidden([g[:, p] for p in parts], [reps[:, p] for p in parts],
                                        [idx[:, p] for p in parts], H, [W[p] for p in parts])
    np.testing.assert_allclose(total, full, rtol=1e-12, atol=1e-12)
