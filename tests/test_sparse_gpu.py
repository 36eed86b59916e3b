"""GPU parity of the sparse forms of reps (csrc/sparse.cu through the C ABI and
sparton_b200.sparse) with the oracle (oracle/sparse_oracle.py, pinned to torch):
bit-exact CSR arrays, top-k values and indices (ties: lower vocab id first), on
the torch fixtures, on seeded SPLADE-like reps of the benchmark shapes, and on
edge cases (empty rows, all-equal rows, k = 1 and k = V, V not a multiple of
the kernels' tiles, NaN, thresholds)."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import sparse_oracle as so
from sparton_b200 import _lib, sparse

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "golden", "sparse_*.npz")))
TORCH = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def splade_like(B, V, dtype, seed, zero_frac=0.5):
    gen = torch.Generator().manual_seed(seed)
    x = torch.log1p(torch.relu(torch.randn(B, V, generator=gen) * 2.0))
    x[torch.rand(B, V, generator=gen) < zero_frac] = 0.0
    return x.to(dtype)


def check(reps_cpu, threshold=0.0, ks=()):
    reps = reps_cpu.cuda()
    x = reps_cpu.float().numpy()
    crow, cols, vals = sparse.csr_arrays(reps, threshold)
    rc, cc, vc = so.csr(x, threshold)
    np.testing.assert_array_equal(crow.cpu().numpy(), rc)
    np.testing.assert_array_equal(cols.cpu().numpy(), cc)
    np.testing.assert_array_equal(vals.float().cpu().numpy(), vc)
    for k in ks:
        v, i = sparse.topk_reps(reps, k)
        rv, ri = so.topk(x, k)
        np.testing.assert_array_equal(v.float().cpu().numpy(), rv)
        np.testing.assert_array_equal(i.cpu().numpy(), ri)


@pytest.mark.parametrize("name", FIXTURES)
def test_fixtures(name):
    c = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    reps = torch.tensor(c["reps"]).to(TORCH[str(c["dtype"])])
    check(reps, float(c["threshold"]), [int(k) for k in c["ks"]])
    r = sparse.nonzero_ratio(reps.cuda()).item()
    assert r == pytest.approx(float(c["nonzero_ratio"]), rel=1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 1), (3, 31), (5, 4096), (4, 4097), (128, 30522),
                                   (2, 250002)], ids=lambda s: "B{}V{}".format(*s))
def test_shapes(dtype, shape):
    B, V = shape
    reps = splade_like(B, V, dtype, seed=B + V)
    ks = sorted({1, min(V, 64), min(V, 256), min(V, 4096)})
    check(reps, 0.0, ks)


def test_edge_rows():
    V = 5000
    reps = torch.zeros(6, V, dtype=torch.bfloat16)
    reps[1] = 1.5                      # all equal
    reps[2, ::7] = 2.0                 # equal values spread over the row
    reps[3, -1] = 9.0                  # only the last column
    reps[4] = splade_like(1, V, torch.bfloat16, seed=3)[0]
    reps[5, 100:140] = torch.arange(40, dtype=torch.float32).to(torch.bfloat16)
    check(reps, 0.0, [1, 2, 17, 715, 4096])
    check(reps, 1.5, [5])
    check(reps, -1.0, [3])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_topk_list_and_row_paths(dtype):
    """Rows whose candidates (entries at or above the k-th largest key's top
    8 bits) overflow the shared-memory list take the row path: all-equal rows,
    rows with fewer nonzeros than k (the k-th largest is 0), signed values;
    and reps whose storage is not 16-byte aligned (scalar first pass)."""
    B, V = 6, 30522
    gen = torch.Generator().manual_seed(11)
    reps = torch.zeros(B, V)
    reps[0] = 1.0                                   # all equal: row path
    reps[1, torch.randperm(V, generator=gen)[:100]] = torch.rand(100, generator=gen) + 0.5
    reps[2] = splade_like(1, V, torch.float32, seed=12)[0]
    reps[3] = torch.randn(V, generator=gen)         # negative and positive
    reps[4, ::3] = 2.0                              # 10174 equals of the top value
    reps[5] = splade_like(1, V, torch.float32, seed=13, zero_frac=0.9)[0]
    reps = reps.to(dtype)
    check(reps, 0.0, [1, 256, 4096])
    # the same rows one element past a 16-byte boundary
    flat = torch.zeros(B * V + 8, dtype=dtype)
    flat[1:1 + B * V] = reps.reshape(-1)
    view = flat.cuda()[1:1 + B * V].view(B, V)
    assert view.data_ptr() % 16 != 0
    x = reps.float().numpy()
    for k in (1, 256, 4096):
        v, i = sparse.topk_reps(view, k)
        rv, ri = so.topk(x, k)
        np.testing.assert_array_equal(v.float().cpu().numpy(), rv)
        np.testing.assert_array_equal(i.cpu().numpy(), ri)
    crow, cols, vals = sparse.csr_arrays(view, 0.0)
    rc, cc, vc = so.csr(x, 0.0)
    np.testing.assert_array_equal(crow.cpu().numpy(), rc)
    np.testing.assert_array_equal(cols.cpu().numpy(), cc)
    np.testing.assert_array_equal(vals.float().cpu().numpy(), vc)


def test_k_zero_and_empty():
    reps = splade_like(3, 100, torch.bfloat16, seed=1).cuda()
    v, i = sparse.topk_reps(reps, 0)
    assert v.shape == (3, 0) and i.shape == (3, 0)
    crow, cols, vals = sparse.csr_arrays(torch.zeros(4, 0, dtype=torch.bfloat16).cuda())
    assert crow.cpu().tolist() == [0] * 5 and cols.numel() == 0
    crow, cols, vals = sparse.csr_arrays(torch.zeros(0, 10, dtype=torch.float16).cuda())
    assert crow.cpu().tolist() == [0]


def test_csr_tensor_and_capi_capacity():
    reps = splade_like(8, 3000, torch.float16, seed=9)
    t = sparse.reps_to_csr(reps.cuda())
    assert t.layout == torch.sparse_csr
    np.testing.assert_array_equal(t.to_dense().cpu().float().numpy(), reps.float().numpy())
    # through the C ABI with too small a capacity: crow complete, the first
    # `capacity` entries written, nothing past them
    lib = _lib.load()
    r = reps.cuda()
    B, V = r.shape
    crow = torch.empty(B + 1, dtype=torch.int64, device="cuda")
    cap = 100
    cols = torch.full((cap + 8,), -1, dtype=torch.int32, device="cuda")
    vals = torch.zeros(cap + 8, dtype=torch.float16, device="cuda")
    ws = torch.zeros(lib.sparton_sparse_workspace_size(B, V), dtype=torch.uint8, device="cuda")
    sh = torch.cuda.current_stream().cuda_stream
    assert lib.sparton_reps_csr(r.data_ptr(), 1, B, V, 0.0, crow.data_ptr(), cols.data_ptr(),
                                vals.data_ptr(), cap, ws.data_ptr(), ws.numel(), sh) == 0
    rc, cc, vc = so.csr(reps.float().numpy())
    np.testing.assert_array_equal(crow.cpu().numpy(), rc)
    np.testing.assert_array_equal(cols[:cap].cpu().numpy(), cc[:cap])
    assert (cols[cap:] == -1).all()
    # invalid k is refused before any launch
    v = torch.empty(B, 1, dtype=torch.float16, device="cuda")
    i = torch.empty(B, 1, dtype=torch.int32, device="cuda")
    assert lib.sparton_reps_topk(r.data_ptr(), 1, B, V, V + 1, v.data_ptr(), i.data_ptr(), sh) != 0
    assert lib.sparton_reps_topk(r.data_ptr(), 1, B, V, 4097, v.data_ptr(), i.data_ptr(), sh) != 0


def test_encode_sparse_with_head():
    from sparton_b200.head import SpartonHead
    from tests._cases import synthetic

    B, S, D, V = 4, 64, 128, 777
    H, W, b, mask, _ = synthetic(B, S, D, V, (8, S), dtype=torch.bfloat16, seed=2, w_std=0.1)
    head = SpartonHead(V, D, use_bias=True).cuda().to(torch.bfloat16)
    head.load({"weight": W, "bias": b})
    with torch.no_grad():
        reps = head(H.cuda(), mask.cuda())
    v, i = sparse.encode_sparse(head, H.cuda(), mask.cuda(), k=32)
    rv, ri = so.topk(reps.float().cpu().numpy(), 32)
    np.testing.assert_array_equal(i.cpu().numpy(), ri)
    t = sparse.encode_sparse(head, H.cuda(), mask.cuda())
    assert torch.equal(t.to_dense(), reps)


def test_rejects_cpu_tensors():
    with pytest.raises(ValueError):
        sparse.topk_reps(torch.rand(2, 3), 1)
