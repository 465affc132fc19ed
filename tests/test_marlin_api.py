"""The Marlin drop-in's host logic on CPU (interface of After-Revision-DROFELL/
operators/core/linear/real_marlin.py and cuda_extends/marlin.py): argument checks,
tuning thresholds, the dense cache and merge."""
import pytest
import torch

from drofell_for_revision_b200.marlin import MarlinDenseCache, MarlinTuningParams, make_marlin_workspace
from drofell_for_revision_b200.real_marlin import MarlinQuantLinear, MarlinQuantLinearMaker


def test_tuning_params():
    with pytest.raises(ValueError):
        MarlinTuningParams(reconstruct_threshold=0)
    tp = MarlinTuningParams()
    assert not tp.use_reconstructed_forward(767, cache_weight=False)
    assert tp.use_reconstructed_forward(768, cache_weight=False)
    assert tp.use_reconstructed_forward(128, cache_weight=True)
    assert not MarlinTuningParams(reconstruct_threshold=None).use_reconstructed_forward(10**6, cache_weight=False)
    assert tp.reuse_reconstruct_cache(True) and not MarlinTuningParams(
        reuse_reconstruct_cache_when_grad=False).reuse_reconstruct_cache(True)


def test_dense_cache():
    c = MarlinDenseCache(torch.device("cpu"))
    with pytest.raises(RuntimeError):
        c.weight(4, 4)
    c.update(8, 16)
    c.update(4, 4)
    c.init_cache()
    assert c.weight(8, 16).shape == (8, 16)
    with pytest.raises(RuntimeError):
        c.weight(16, 16)
    with pytest.raises(RuntimeError):
        c.update(32, 32)
    with pytest.raises(RuntimeError):
        c.init_cache()


def test_workspace_needs_cuda():
    with pytest.raises(ValueError):
        make_marlin_workspace(torch.device("cpu"))


def test_linear_checks_and_buffers():
    with pytest.raises(ValueError):
        MarlinQuantLinear(128, 256, 256, True, False)  # no bias in the Marlin backend
    with pytest.raises(ValueError):
        MarlinQuantLinear(128, 250, 256, False, False)
    with pytest.raises(ValueError):
        MarlinQuantLinear(96, 256, 256, False, False)  # group size does not divide K
    m = MarlinQuantLinear(-1, 256, 64, False, True)
    assert m.group_size == 256 and not m.use_act_order  # full-K group: no act-order
    sd = m.state_dict()
    assert set(sd) == {"qweight", "qzeros", "scales", "g_idx"}  # the workspace is not persistent
    assert sd["qweight"].shape == (32, 64) and sd["qzeros"].shape == (1, 8) and sd["scales"].dtype == torch.float16
    with pytest.raises(RuntimeError):
        m(torch.zeros(1, 256))  # not finished by post_init


def test_maker_merge():
    mk = MarlinQuantLinearMaker(64, False)
    a, b = mk.make_linear(256, 64), mk.make_linear(256, 96)
    a.qweight.fill_(1)
    b.qweight.fill_(2)
    merged = mk.merge([a, b])
    assert merged.outfeatures == 160 and mk.quant_linears == [merged]
    assert torch.equal(merged.qweight[:, :64], a.qweight) and torch.equal(merged.qweight[:, 64:], b.qweight)
    assert merged.qzeros.shape == (4, 20) and merged.scales.shape == (4, 160)
    with pytest.raises(ValueError):
        mk.merge([])
    c = mk.make_linear(512, 64)
    with pytest.raises(ValueError):
        mk.merge([merged, c])
    with pytest.raises(RuntimeError):
        MarlinQuantLinearMaker(64, False).post_init(MarlinTuningParams(), MarlinDenseCache(torch.device("cpu")))
