"""Host-side logic of the drop-in: buffer layout, act-order permutation, sharding."""
import numpy as np
import pytest
import torch

from drofell_for_revision_b200 import exllama, real_quant, sharded, synthetic
from oracle import w4a16_oracle as orc


def test_quantlinear_buffers_match_reference_layout():
    # real_quant.py:25-49: qweight [K/32*4, N], qzeros [ceil(K/g), N/32*4], scales [ceil(K/g), N], g_idx k//g
    ql = real_quant.QuantLinear(128, 4096, 11008, True, False)
    assert ql.qweight.shape == (512, 11008) and ql.qweight.dtype == torch.int32
    assert ql.qzeros.shape == (32, 1376) and ql.qzeros.dtype == torch.int32
    assert ql.scales.shape == (32, 11008) and ql.scales.dtype == torch.float16
    assert ql.g_idx.dtype == torch.int32 and int(ql.g_idx[300]) == 2
    assert ql.bias.shape == (11008,) and ql.bias.dtype == torch.float16
    names = [n for n, _ in ql.named_buffers()]
    assert names == ["qweight", "qzeros", "scales", "g_idx", "bias"]


def test_quantlinear_asserts_like_reference():
    with pytest.raises(AssertionError):
        real_quant.QuantLinear(128, 100, 64, False, False)
    with pytest.raises(AssertionError):
        real_quant.QuantLinear(128, 4096, 100, False, False)
    ql = real_quant.QuantLinear(-1, 256, 64, False, False)
    assert ql.group_size == 256 and ql.qzeros.shape == (1, 8)


def test_quantlinear_post_init_requires_cuda():
    ql = real_quant.QuantLinear(128, 256, 64, False, False)
    with pytest.raises(AssertionError):
        ql.post_init(exllama.TuningParams(), exllama.CacheV2(torch.device("cpu")))


def test_maker_tracks_linears():
    mk = real_quant.QuantLinearMaker(128, False)
    a = mk.make_linear(256, 64)
    b = mk.make_linear(256, 128, bias=True)
    assert mk.quant_linears == [a, b] and a.bias is None and b.bias is not None


def test_tuning_params_defaults_match_reference():
    tp = exllama.TuningParams()
    assert tp.BLOCK_KN_SIZE == 128 and tp.BLOCK_M_SIZE_MAX == 8 and tp.MATMAL_RECONSTRUCT_THRESHOLD_V2 == 50


def test_cache_v2_semantics():
    c = exllama.CacheV2(torch.device("cpu"))
    c.update_temp_weight_size(10)
    c.update_temp_weight_size(5)
    assert c.temp_weight_size == 10 and not c.cache_created
    with pytest.raises(AssertionError):
        _ = c.temp_weight
    c.init_cache()
    assert c.temp_weight.shape == (1, 10)


def test_act_order_permutation_matches_reference_x_map():
    layer = synthetic.make_layer(512, 64, 128, act_order=True, seed=3)
    perm_np = orc.act_order_perm(layer.g_idx.numpy(), 4)
    perm_t = torch.argsort(layer.g_idx.to(torch.int64), stable=True).to(torch.int32).numpy()
    np.testing.assert_array_equal(perm_np, perm_t)
    # every group has exactly group_size members
    assert np.all(np.bincount(layer.g_idx.numpy()) == 128)


def test_synthetic_distributions():
    layer = synthetic.make_layer(1024, 256, 128, seed=0)
    q = orc.unpack_qweight(layer.qweight.numpy())
    z = orc.unpack_qzeros(layer.qzeros.numpy())
    assert q.min() == 0 and q.max() == 15 and abs(q.mean() - 7.5) < 0.1
    assert z.min() == 1 and z.max() == 16
    s = layer.scales.float().numpy()
    assert s.min() >= 1e-3 - 1e-6 and 0.015 < s.mean() < 0.03
    # deterministic
    again = synthetic.make_layer(1024, 256, 128, seed=0)
    assert torch.equal(layer.qweight, again.qweight)


def test_shard_columns_reassemble():
    layer = synthetic.make_layer(256, 256, 64, seed=1)
    W = orc.dequant_fp16(layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(), group_size=64)
    parts = []
    for r in range(4):
        qw, qz, sc = sharded.shard_columns(layer.qweight, layer.qzeros, layer.scales, r, 4)
        parts.append(orc.dequant_fp16(qw.numpy(), qz.numpy(), sc.numpy(), group_size=64))
    np.testing.assert_array_equal(np.concatenate(parts, 1).view(np.uint16), W.view(np.uint16))
    with pytest.raises(ValueError):
        sharded.shard_bounds(256, 0, 3)
    with pytest.raises(ValueError):
        sharded.shard_bounds(64, 0, 4)  # 16 columns per rank < 32
