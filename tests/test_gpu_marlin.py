"""The Marlin drop-in (symmetric GPTQ: every stored zero nibble 7, z = 8) on the B200
kernels, against the oracle. The reference's Marlin dequant is (q - 8) * s
(After-Revision-DROFELL/cuda_extends/marlin/marlin_dequant.cu:70-72), the GPTQ formula
of real_quant.py:69-90 with every zero point 8, which the oracle evaluates. Tolerance
max|Y - Y_ref| / max|Y_ref| <= 1e-2 (north star); dequant bit-exact."""
import numpy as np
import pytest
import torch

from drofell_for_revision_b200 import _capi, synthetic
from drofell_for_revision_b200.marlin import MarlinDenseCache, MarlinTuningParams
from drofell_for_revision_b200.real_marlin import MarlinQuantLinearMaker
from oracle import w4a16_oracle as orc

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
TOL = 1e-2


def _sym_layer(K, N, g=128, act=False, seed=0):
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=seed)
    layer.qzeros.fill_(0x77777777)
    return layer


def _load(maker, layer):
    lin = maker.make_linear(layer.K, layer.N)
    lin.qweight.copy_(layer.qweight)
    lin.qzeros.copy_(layer.qzeros)
    lin.scales.copy_(layer.scales)
    lin.g_idx.copy_(layer.g_idx)
    return lin


def _ref(layer, x):
    return orc.w4a16_linear_ref(x.float().half().numpy(), layer.qweight.numpy(), layer.qzeros.numpy(),
                                layer.scales.numpy(), layer.g_idx.numpy() if layer.act_order else None,
                                layer.group_size)


@pytest.mark.parametrize("act", [False, True])
@pytest.mark.parametrize("M", [1, 2, 8, 40, 300])
def test_marlin_linear_forward(act, M):
    K, N = 2048, 1536
    layer = _sym_layer(K, N, act=act, seed=K + M)
    mk = MarlinQuantLinearMaker(128, act)
    lin = _load(mk, layer).to(DEV)
    mk.post_init(MarlinTuningParams(), MarlinDenseCache(DEV))
    assert lin.q4_matrix._h.symmetric
    x = synthetic.make_activations(M, K, seed=M)
    y = lin(x.to(DEV))
    assert y.dtype == torch.float16 and y.shape == (M, N)
    assert orc.rel_err(y.float().cpu().numpy(), _ref(layer, x)) < TOL
    w = lin.reconstruct_weight(torch.empty((K, N), dtype=torch.float16, device=DEV))
    ref = orc.dequant_fp16(layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(),
                           layer.g_idx.numpy() if act else None, 128)
    np.testing.assert_array_equal(w.cpu().view(torch.int16).numpy().view(np.uint16), ref.view(np.uint16))


def test_marlin_merged_qkv_bf16_input_and_backward():
    """q / k / v merged by the maker (real_loader_marlin.py:65-79), a bf16 input cast to
    fp16 and back (real_marlin.py:139-157), and the input gradient."""
    K = 1024
    parts = [_sym_layer(K, n, seed=i) for i, n in enumerate((1024, 256, 256))]
    mk = MarlinQuantLinearMaker(128, False)
    lins = [_load(mk, l) for l in parts]
    merged = mk.merge(lins).to(DEV)
    mk.post_init(MarlinTuningParams(), MarlinDenseCache(DEV))
    x = synthetic.make_activations(6, K, seed=3).to(torch.bfloat16)
    xd = x.to(DEV).requires_grad_(True)
    y = merged(xd)
    assert y.dtype == torch.bfloat16 and y.shape == (6, 1536)
    ref = np.concatenate([_ref(l, x) for l in parts], axis=1)
    assert orc.rel_err(y.float().detach().cpu().numpy(), ref) < TOL
    gy = synthetic.make_activations(6, 1536, seed=4).to(torch.bfloat16).to(DEV)
    y.backward(gy)
    W = np.concatenate([orc.dequant_fp16(l.qweight.numpy(), l.qzeros.numpy(), l.scales.numpy(), None, 128)
                        for l in parts], axis=1).astype(np.float32)
    gref = gy.float().cpu().numpy() @ W.T
    assert xd.grad.dtype == torch.bfloat16
    assert orc.rel_err(xd.grad.float().cpu().numpy(), gref) < TOL


def test_marlin_rejects_asymmetric_zero_points():
    layer = synthetic.make_layer(256, 128, 128, seed=5)  # random zero points
    mk = MarlinQuantLinearMaker(128, False)
    _load(mk, layer).to(DEV)
    with pytest.raises(ValueError, match="symmetric"):
        mk.post_init(MarlinTuningParams(), MarlinDenseCache(DEV))


@pytest.mark.parametrize("path", [_capi.PATH_GEMV, _capi.PATH_TC])
@pytest.mark.parametrize("M", [1, 5, 200])
def test_symmetric_fast_path(path, M):
    """A handle over zero points that are all 8 finds that at creation and runs every
    kernel without loading them: GEMV, tcgen05 GEMM and the transposed GEMM against the
    oracle. One other zero nibble anywhere keeps the loads."""
    K, N = 4096, 1024
    layer = _sym_layer(K, N, seed=M)
    h = _capi.Handle(layer.qweight.to(DEV), layer.qzeros.to(DEV), layer.scales.to(DEV), None, 0)
    assert h.symmetric
    x = synthetic.make_activations(M, K, seed=M + 9)
    y = torch.empty((M, N), dtype=torch.float16, device=DEV)
    h.gemm(x.to(DEV), y, path)
    dy = synthetic.make_activations(M, N, seed=M + 10)
    dx = torch.empty((M, K), dtype=torch.float16, device=DEV)
    h.gemm_t(dy.to(DEV), dx)
    torch.cuda.synchronize()
    assert orc.rel_err(y.float().cpu().numpy(), _ref(layer, x)) < 4e-3
    W = orc.dequant_fp16(layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(), None, 128)
    assert orc.rel_err(dx.float().cpu().numpy(), dy.float().numpy() @ W.astype(np.float32).T) < 2e-3
    qz = layer.qzeros.clone()
    qz[-1, -1] = 0x77777776
    h2 = _capi.Handle(layer.qweight.to(DEV), qz.to(DEV), layer.scales.to(DEV), None, 0)
    assert not h2.symmetric
