"""Parity at the full BASELINE shapes (configs 2-5), forward and backward,
through the torch ops (C ABI underneath), against the CPU oracle on samples.

A full [B,S,V] oracle is out of reach at these sizes (config 5's logits would
be 64*1024*128256 fp64 values), so every config is checked three ways:

* sampled vocab columns (~200: random ones, the ragged last vocab tile, the
  first and last columns): reps and idx against ``orc.forward`` on those
  columns of W (rtol 1e-2, argmax exact outside near-ties, whose count is
  reported), dW and db against the fused-backward formula on the same columns;
* sampled hidden rows: dH[b, s, :] for a few (b, s) per sampled batch row (the
  heaviest bucket, position 0, the last valid position, a random valid one, a
  padded one) against the sum over the vocab ids whose argmax is s, computed
  in fp64 from the kernel's own reps / idx (sparton_kernel.py:531-561);
* size-independent properties on every element: reps >= 0, idx inside the
  row, reps == 0 => idx == 0, dH == 0 at padded positions, and the backward
  bit-identical when run twice (no atomics).

Configs: 2 = B128 S256 D768 V30522 bf16; 3 = B32 S256 D768
V250002 bf16; 4 = B512 S512 D768 V30522 fp16, 10% of rows full length;
5 = B64 S1024 D4096 V128256 bf16, no bias, W ~ N(0, 0.01).
"""
import numpy as np
import pytest
import torch

import sparton_b200.ops  # noqa: F401
from oracle import sparton_oracle as orc
from tests._cases import np64, synthetic

pytestmark = pytest.mark.gpu

CONFIGS = {
    "config2": dict(B=128, S=256, D=768, V=30522, dtype=torch.bfloat16, lengths=(32, 256),
                    bias=True, w_std=0.02, full_frac=0.0),
    "config3": dict(B=32, S=256, D=768, V=250002, dtype=torch.bfloat16, lengths=(32, 256),
                    bias=True, w_std=0.02, full_frac=0.0),
    "config4": dict(B=512, S=512, D=768, V=30522, dtype=torch.float16, lengths=(64, 512),
                    bias=True, w_std=0.02, full_frac=0.1),
    "config5": dict(B=64, S=1024, D=4096, V=128256, dtype=torch.bfloat16, lengths=(256, 1024),
                    bias=False, w_std=0.01, full_frac=0.0),
}
RTOL = 1e-2


def sample_columns(V, rng, n=170):
    tail = np.arange(max(0, V - 24), V)          # the ragged last vocab tile(s)
    edge = np.array([0, 1, 127, 128, V // 2])    # first tiles, a tile boundary
    return np.unique(np.concatenate([rng.choice(V, min(n, V), replace=False), tail, edge]))


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_full_size_parity(name, record_property):
    c = CONFIGS[name]
    B, S, D, V = c["B"], c["S"], c["D"], c["V"]
    H, W, b, mask, g = synthetic(B, S, D, V, c["lengths"], dtype=c["dtype"], use_bias=c["bias"],
                                 w_std=c["w_std"], seed=0, full_frac=c["full_frac"])
    dev = torch.device("cuda")
    Hd, Wd, md, gd = H.to(dev), W.to(dev), mask.to(dev), g.to(dev)
    bd = b.to(dev) if b is not None else None
    reps, idx = torch.ops.sparton.fused_sparton_fwd(Hd, Wd, bd, md)
    dH, dW, db = torch.ops.sparton.fused_sparton_bwd(gd, reps, idx, Hd, Wd, bd, md)
    dH2, dW2, db2 = torch.ops.sparton.fused_sparton_bwd(gd, reps, idx, Hd, Wd, bd, md)
    torch.cuda.synchronize()
    assert torch.equal(dH, dH2) and torch.equal(dW, dW2) and torch.equal(db, db2), \
        "backward not deterministic"
    del dH2, dW2, db2

    # -- properties on every element
    L = mask.sum(1).to(dev)
    assert bool((reps >= 0).all())
    assert bool((idx >= 0).all()) and bool((idx < L[:, None].clamp(min=1)).all())
    assert bool(((reps == 0) <= (idx == 0)).all())
    assert bool((dH[md == 0] == 0).all()), "nonzero d_hidden at a padded position"
    assert bool(torch.isfinite(dH).all()) and bool(torch.isfinite(dW).all())

    reps_c, idx_c = reps.cpu(), idx.cpu()
    rng = np.random.default_rng(1)
    sel = sample_columns(V, rng)
    sel_t = torch.tensor(sel)
    mask_np = mask.numpy()
    H64 = np64(H)

    # -- forward on sampled columns
    Wsel, bsel = np64(W[sel_t]), (np64(b[sel_t]) if b is not None else None)
    ref, ref_idx, _ = orc.forward(H64, Wsel, bsel, mask_np)
    np.testing.assert_allclose(np64(reps_c[:, sel_t]), ref, rtol=RTOL, atol=1e-3,
                               err_msg=f"{name} reps")
    ours_idx = idx_c[:, sel_t].numpy()
    ok = orc.accept_indices(ours_idx, H64, Wsel, bsel, mask_np)
    assert ok.all(), f"{name}: {int((~ok).sum())} argmax mismatches outside near-ties"
    near = int(orc.near_tie_mask(H64, Wsel, bsel, mask_np).sum())
    differ = int((ours_idx != ref_idx).sum())
    record_property("near_ties", near)
    record_property("idx_differing_at_near_ties", differ)
    print(f"{name}: {len(sel)} sampled columns x {B} rows, near-ties {near}, "
          f"idx differing from the oracle (all at near-ties) {differ}")

    # -- dW / db on sampled columns (fused-backward formula on our reps / idx)
    g64, r64 = np64(g), np64(reps_c)
    gp = np.where(r64 > 0, g64 * np.exp(-r64), 0.0)          # [B, V]
    gp_sel = gp[:, sel]
    rows = H64[np.arange(B)[:, None], ours_idx]             # [B, n, D]
    dW_ref = np.einsum("bn,bnd->nd", gp_sel, rows)
    dW_sel = np64(dW[sel_t.to(dev)].cpu())
    atol_w = RTOL * 1e-2 * np.abs(dW_ref).max()
    np.testing.assert_allclose(dW_sel, dW_ref, rtol=RTOL, atol=atol_w, err_msg=f"{name} dW")
    if b is not None:
        db_ref = gp_sel.sum(0)
        np.testing.assert_allclose(np64(db[sel_t.to(dev)].cpu()), db_ref, rtol=RTOL,
                                   atol=RTOL * 1e-2 * np.abs(db_ref).max(), err_msg=f"{name} db")
    else:
        assert db.numel() == 0

    # -- dH on sampled (b, s) rows
    idx_np = idx_c.numpy()
    Lnp = mask_np.sum(1)
    checked = 0
    for bb in rng.choice(B, 4, replace=False):
        counts = np.bincount(idx_np[bb][r64[bb] > 0], minlength=S)
        cand = {int(np.argmax(counts)), 0, max(int(Lnp[bb]) - 1, 0),
                int(rng.integers(0, max(int(Lnp[bb]), 1)))}
        if Lnp[bb] < S:
            cand.add(S - 1)                                   # padded: must be 0
        for s in sorted(cand):
            vs = np.nonzero((idx_np[bb] == s) & (r64[bb] > 0))[0]
            ref_row = gp[bb, vs] @ np64(W[torch.tensor(vs, dtype=torch.long)]) if len(vs) else \
                np.zeros(D)
            ours = np64(dH[bb, s].cpu())
            atol_h = RTOL * 1e-2 * max(np.abs(ref_row).max(), 1e-30) + 1e-30
            np.testing.assert_allclose(ours, ref_row, rtol=RTOL, atol=atol_h,
                                       err_msg=f"{name} dH[{bb},{s}] ({len(vs)} entries)")
            checked += 1
    record_property("dH_rows_checked", checked)
