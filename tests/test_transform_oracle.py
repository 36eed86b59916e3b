"""The MLM-transform oracle (oracle/transform_oracle.py) against fixtures made
by running the reference's own _get_backbone_and_head and ProjectionPyTorch on
small random-init BERT and RoBERTa models (tests/golden/make_golden_transform.py),
float64: reps and every gradient to 1e-9."""
import glob
import os

import numpy as np
import pytest

from oracle import transform_oracle as to

HERE = os.path.dirname(os.path.abspath(__file__))
NAMES = sorted(os.path.basename(p)[:-4]
               for p in glob.glob(os.path.join(HERE, "golden", "transform_*.npz")))


def test_fixtures_exist():
    assert len(NAMES) >= 2


@pytest.mark.parametrize("name", NAMES)
def test_transform_oracle_matches_reference(name):
    c = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    reps, grads, _ = to.projection(c["x"], c["Wd"], c["bd"], c["gamma"], c["beta"],
                                   float(c["eps"]), c["W"], c["b"], c["mask"], c["g"])
    np.testing.assert_allclose(reps, c["reps"], rtol=1e-9, atol=1e-12)
    for k in ("dx", "dWd", "dbd", "dgamma", "dbeta", "dW", "db"):
        ref = c[k]
        np.testing.assert_allclose(grads[k], ref, rtol=1e-9, atol=1e-9 * max(np.abs(ref).max(), 1.0),
                                   err_msg=k)


def test_rounding_helper():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9, -2.5, 1e-3])
    np.testing.assert_array_equal(to.round_to(x, "bfloat16")[:3], [1.0, 1.0, 1.0 + 2 ** -7])
    np.testing.assert_array_equal(to.round_to(x, "float16"), x.astype(np.float16))
