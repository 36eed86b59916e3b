"""The sparse-form oracle (oracle/sparse_oracle.py) against fixtures made by
torch (tests/golden/make_golden_sparse.py): CSR arrays exactly, top-k values
exactly, top-k indices pointing at those values, and the nonzero ratio."""
import glob
import os

import numpy as np
import pytest

from oracle import sparse_oracle as so

HERE = os.path.dirname(os.path.abspath(__file__))
NAMES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "golden", "sparse_*.npz")))


def test_fixtures_exist():
    assert len(NAMES) >= 3


@pytest.mark.parametrize("name", NAMES)
def test_sparse_oracle_matches_torch_fixture(name):
    c = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    reps = c["reps"]
    crow, cols, vals = so.csr(reps, float(c["threshold"]))
    np.testing.assert_array_equal(crow, c["crow"])
    np.testing.assert_array_equal(cols, c["cols"])
    np.testing.assert_array_equal(vals, c["vals"])
    for k in c["ks"]:
        v, i = so.topk(reps, int(k))
        np.testing.assert_array_equal(v, c[f"topk{k}"])  # NaN == NaN in assert_array_equal
        got = np.take_along_axis(reps, i, axis=1)
        np.testing.assert_array_equal(got, v)
        assert all(len(set(row)) == len(row) for row in i)
    assert so.nonzero_ratio(reps) == pytest.approx(float(c["nonzero_ratio"]), rel=1e-6)


def test_topk_ties_take_lower_ids():
    x = np.array([[1.0, 3.0, 3.0, 0.0, 3.0, 2.0]])
    v, i = so.topk(x, 3)
    assert i.tolist() == [[1, 2, 4]] and v.tolist() == [[3.0, 3.0, 3.0]]
    v, i = so.topk(x, 2)
    assert i.tolist() == [[1, 2]]
