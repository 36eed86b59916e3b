"""Host logic of the transform and sparse modules (no GPU): which transform
modules are accepted, parameter sharing and weight tying of SpartonProjection,
and the CUDA-only checks."""
import pytest
import torch
from torch import nn

from sparton_b200 import sparse
from sparton_b200 import transform as tr


class BertLike(nn.Module):  # BertPredictionHeadTransform's attribute names
    def __init__(self, act):
        super().__init__()
        self.dense = nn.Linear(16, 16)
        self.transform_act_fn = act
        self.LayerNorm = nn.LayerNorm(16, eps=1e-12)


class RobertaLike(nn.Module):  # the reference's RobertaTransform (model.py:25-35)
    def __init__(self):
        super().__init__()
        self.dense = nn.Linear(16, 16)
        self.layer_norm = nn.LayerNorm(16)


def test_from_module_accepts_bert_and_roberta_layouts():
    b = BertLike(nn.GELU())
    t = tr.MLMTransform.from_module(b)
    assert t.dense is b.dense and t.layer_norm is b.LayerNorm  # parameters shared
    r = RobertaLike()
    t = tr.MLMTransform.from_module(r)
    assert t.dense.weight is r.dense.weight and t.layer_norm.bias is r.layer_norm.bias


def test_from_module_accepts_transformers_gelu():
    transformers = pytest.importorskip("transformers")
    act = transformers.activations.ACT2FN["gelu"]
    assert tr._is_exact_gelu(act)
    assert not tr._is_exact_gelu(transformers.activations.ACT2FN["gelu_new"])
    assert not tr._is_exact_gelu(nn.ReLU())


@pytest.mark.parametrize("act", [nn.GELU(approximate="tanh"), nn.ReLU(), nn.SiLU()])
def test_from_module_rejects_other_activations(act):
    with pytest.raises(ValueError):
        tr.MLMTransform.from_module(BertLike(act))


def test_rejects_unknown_transform_and_bad_layer_norm():
    with pytest.raises(ValueError):
        tr.MLMTransform.from_module(nn.Linear(16, 16))
    with pytest.raises(ValueError):
        tr.MLMTransform(nn.Linear(16, 16), nn.LayerNorm(8))
    with pytest.raises(ValueError):
        tr.MLMTransform(nn.Linear(16, 16), nn.LayerNorm(16, elementwise_affine=False))


def test_projection_ties_decoder():
    decoder = nn.Linear(16, 50)
    proj = tr.SpartonProjection(RobertaLike(), decoder)
    assert proj.sparton_head.weight is decoder.weight and proj.sparton_head.bias is decoder.bias
    assert proj.sparton_head.vocab_size == 50 and proj.sparton_head.hidden_dim == 16


def test_cuda_only():
    with pytest.raises(ValueError):
        tr.transform_fwd_impl(torch.rand(4, 16), torch.ones(16), torch.zeros(16), 1e-5)
    with pytest.raises(ValueError):
        sparse.reps_to_csr(torch.rand(2, 3))
    with pytest.raises(ValueError):
        sparse.nonzero_ratio(torch.rand(2, 3))
