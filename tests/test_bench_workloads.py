"""The bench's workloads against BASELINE.json's configs (CPU): shapes, dtype,
length ranges, bias, weight scale, and the synthetic inputs' properties."""
import json
import os
import re

import pytest
import torch

import bench

HERE = os.path.dirname(os.path.abspath(__file__))
CONFIGS = json.load(open(os.path.join(HERE, "..", "BASELINE.json")))["configs"]


def _num(text, name):
    m = re.search(rf"\b{name}=(\d+)", text)
    return int(m.group(1)) if m else None


@pytest.mark.parametrize("i", [1, 2, 3, 4])
def test_workload_matches_baseline_config(i):
    text = CONFIGS[i]
    c = bench.WORKLOADS[f"config{i + 1}"]
    for k in ("B", "S", "D", "V"):
        assert c[k] == _num(text, k), (i, k)
    dtype = "fp16" if "fp16" in text else "bf16"
    assert c["dtype"] == {"fp16": torch.float16, "bf16": torch.bfloat16}[dtype]
    lo, hi = map(int, re.search(r"uniform in \[(\d+),\s*(\d+)\]", text).groups())
    assert c["lengths"] == (lo, hi)
    assert c["bias"] == ("no bias" not in text)
    if "N(0,0.01)" in text:
        assert c["w_std"] == 0.01
    if "10% of rows full length" in text:
        assert c["full_frac"] == 0.1


def test_default_is_the_metric_config():
    assert bench.CFG is bench.WORKLOADS["config2"]


def test_synthetic_inputs_follow_the_config():
    c = dict(bench.WORKLOADS["config4"], B=200, S=64, D=16, V=8, lengths=(10, 64))
    H, W, b, mask, g, L = bench.make_inputs(c)
    assert H.shape == (200, 64, 16) and W.shape == (8, 16) and g.shape == (200, 8)
    assert H.dtype == torch.float16 and b is not None
    assert torch.equal(mask.sum(1), L) and (L >= 10).all() and (L <= 64).all()
    assert (L == 64).float().mean() > 0.05  # the full-length fraction of config 4
    again = bench.make_inputs(c)
    assert torch.equal(H, again[0]) and torch.equal(L, again[5])  # seeded


def test_cpu_baseline_runs_the_whole_batch_when_it_fits():
    c = dict(bench.WORKLOADS["config2"], B=4, S=16, D=32, V=64, lengths=(2, 16))
    assert bench.cpu_rows_for(c) == 4  # a few KB per row: the whole batch
    res = bench.cpu_baseline(c, bench.cpu_rows_for(c), steps=1, warmup=1)
    assert res["kind"] == "port" and not res["extrapolated"] and res["value"] > 0
    assert "whole batch" in res["sample"] and res["cpu_model"]
    part = bench.cpu_baseline(c, 2, steps=1, warmup=1)
    assert part["extrapolated"] and "extrapolated" in part["sample"]
