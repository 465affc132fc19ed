"""The two bindings of the forward, through QuantLinear: the C++ torch fast path
(_w4a16_torch) and the ctypes path (_capi.Handle.gemm) run the same kernels and must
agree bit for bit; workspaces a captured CUDA graph uses survive later growth."""
import numpy as np
import pytest
import torch

from drofell_for_revision_b200 import _capi, exllama, real_quant, synthetic
from oracle import w4a16_oracle as orc

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
TOL = 1e-2


def _ql(layer, bias=None):
    m = real_quant.QuantLinear(layer.group_size, layer.K, layer.N, bias is not None, layer.act_order)
    m.qweight.copy_(layer.qweight)
    m.qzeros.copy_(layer.qzeros)
    m.scales.copy_(layer.scales)
    m.g_idx.copy_(layer.g_idx)
    if bias is not None:
        m.bias.copy_(bias)
    m = m.to(DEV)
    m.post_init(exllama.TuningParams(), exllama.CacheV2(DEV))
    return m


def test_fast_path_is_built_and_used():
    assert _capi.torch_fast_path() is not None


@pytest.mark.parametrize("act", [False, True])
@pytest.mark.parametrize("shape", [(1,), (2, 3), (64,), (2, 150)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fast_path_matches_ctypes_path(act, shape, dtype):
    layer = synthetic.make_layer(2048, 1536, 128, act_order=act, seed=7)
    bias = (torch.randn(1536) * 0.1).half()
    m = _ql(layer, bias)
    x = synthetic.make_activations(int(np.prod(shape)), 2048, seed=3, dtype=dtype).view(*shape, 2048).to(DEV)
    y_fast = m(x)
    y_ct = m.q4_matrix.matmul(x, None, None)
    y_ct += m.bias
    torch.cuda.synchronize()
    assert y_fast.shape == (*shape, 1536) and y_fast.dtype == dtype
    assert torch.equal(y_fast, y_ct)
    dt = "bf16" if dtype == torch.bfloat16 else "fp16"
    x2 = x.view(-1, 2048).cpu()
    xin = x2.view(torch.int16).numpy().view(np.uint16) if dt == "bf16" else x2.numpy()
    ref = orc.w4a16_linear_ref(xin, layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(),
                               layer.g_idx.numpy() if act else None, 128, dtype=dt) + bias.float().numpy()
    assert orc.rel_err(y_fast.float().cpu().numpy().reshape(-1, 1536), ref) < TOL


@pytest.mark.parametrize("binding", ["fast", "ctypes"])
def test_workspace_growth_keeps_captured_graphs_valid(binding):
    """Capture at a small M (act-order: the X gather needs workspace), grow the workspace
    with an eager call at a much larger M, then replay the graph: it still writes into
    the workspace it captured, which the handle has kept alive."""
    layer = synthetic.make_layer(4096, 1024, 128, act_order=True, seed=11)
    m = _ql(layer)

    def fwd(x):
        if binding == "fast":
            return m(x)
        out = torch.empty((x.shape[0], 1024), dtype=torch.float16, device=DEV)
        m.q4_matrix._h.gemm(x, out)
        return out

    xs = synthetic.make_activations(2, 4096, seed=1).to(DEV)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fwd(xs)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        y_small = fwd(xs)
    big = synthetic.make_activations(3000, 4096, seed=2).to(DEV)  # grows the workspace (gather + split)
    y_big = fwd(big)
    filler = torch.full((64 << 20,), 7, dtype=torch.uint8, device=DEV)  # reuse any freed memory
    g.replay()
    torch.cuda.synchronize()
    del filler
    args = (layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(), layer.g_idx.numpy(), 128)
    assert orc.rel_err(y_small.float().cpu().numpy(), orc.w4a16_linear_ref(xs.cpu().numpy(), *args)) < TOL
    cols = np.concatenate([np.arange(b, b + 8) for b in range(0, 1024, 128)])  # 8-column blocks
    ref_big = orc.w4a16_linear_ref(big.cpu().numpy(), layer.qweight.numpy()[:, cols],
                                   layer.qzeros.numpy()[:, np.unique(cols // 8)], layer.scales.numpy()[:, cols],
                                   layer.g_idx.numpy(), 128)
    assert orc.rel_err(y_big[:, cols].float().cpu().numpy(), ref_big) < TOL
    del g
