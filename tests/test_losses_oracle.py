"""The loss oracle (oracle/losses_oracle.py) against fixtures made by running
the reference's own training losses (tests/golden/make_golden_losses.py)."""
import glob
import os

import numpy as np
import pytest

from oracle import losses_oracle as lo

HERE = os.path.dirname(os.path.abspath(__file__))
NAMES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "golden", "losses_*.npz")))
# Fixture values were computed by the reference in the fixture's dtype. In
# bf16 the reference rounds the scores, the softmax and every gradient product
# to 8 significant bits, so the bf16 case is held to 5% of the largest entry.
RTOL = {"float64": 1e-10, "float32": 1e-4, "bfloat16": 5e-2}


def test_fixtures_exist():
    assert len(NAMES) >= 3


@pytest.mark.parametrize("name", NAMES)
def test_loss_oracle_matches_reference_fixture(name):
    c = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    rtol = RTOL[str(c["dtype"])]
    q, d, t = c["q"], c["d"], float(c["temperature"])
    nce, dq, dd = lo.info_nce(q, d, t)
    np.testing.assert_allclose(nce, c["nce"], rtol=rtol)
    scale = max(np.abs(c["nce_dq"]).max(), 1e-30)
    np.testing.assert_allclose(dq, c["nce_dq"], rtol=rtol, atol=rtol * scale)
    np.testing.assert_allclose(dd, c["nce_dd"], rtol=rtol, atol=rtol * np.abs(c["nce_dd"]).max())
    v, g = lo.l1(q)
    np.testing.assert_allclose(v, c["l1"], rtol=rtol)
    np.testing.assert_allclose(g, c["l1_dq"], rtol=rtol, atol=1e-12)
    v, g = lo.flops(q)
    np.testing.assert_allclose(v, c["flops"], rtol=rtol)
    np.testing.assert_allclose(g, c["flops_dq"], rtol=rtol, atol=rtol * np.abs(c["flops_dq"]).max())


def test_sharded_scores_equal_full_scores():
    rng = np.random.default_rng(0)
    q, d = rng.random((5, 301)), rng.random((7, 301))
    cuts = [0, 100, 128, 301]
    qs = [q[:, a:b] for a, b in zip(cuts, cuts[1:])]
    ds = [d[:, a:b] for a, b in zip(cuts, cuts[1:])]
    np.testing.assert_allclose(lo.sharded_scores(qs, ds), q @ d.T, rtol=1e-12)
