"""w4a16_gemm_static (fixed device scratch, no allocation) against w4a16_gemm.

Collected last on purpose: it must pass both alone in a fresh process (the first
call looks up the scratch array's address) and after every other test has used the
library on the same device.
"""
import pytest
import torch

from drofell_for_revision_b200 import _capi, synthetic
from oracle import w4a16_oracle as orc

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
TOL_TC = 2e-3    # the tcgen05 paths' tolerance in test_gpu_parity.py
TOL_GEMV = 4e-3  # the GEMV tolerance in test_gpu_parity.py


def _handle(layer):
    return _capi.Handle(layer.qweight.to(DEV), layer.qzeros.to(DEV), layer.scales.to(DEV),
                        layer.g_idx if layer.act_order else None, 0)


# every case needs scratch: the act-order X gather, or split-K partial tiles
@pytest.mark.parametrize("K,N,g,act,M,path,tol", [
    (1024, 1024, 128, True, 1, _capi.PATH_AUTO, TOL_GEMV),       # GEMV + act-order gather
    (4096, 1024, 128, True, 12, _capi.PATH_TC, TOL_TC),          # exact-W GEMM at a decode size + gather
    (11008, 256, 128, False, 64, _capi.PATH_TC_EXACT, TOL_TC),   # exact-W GEMM, split-K partials
    (2048, 512, 64, True, 200, _capi.PATH_AUTO, TOL_TC),         # exact-W GEMM, gather + split-K
])
def test_static_scratch_matches_workspace_entry_point(K, N, g, act, M, path, tol):
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=K + 3 * N + M)
    h = _handle(layer)
    x = synthetic.make_activations(M, K, seed=M + 1).to(DEV)
    assert h.workspace_size(M, torch.float16, path) > 0  # the case really uses scratch
    y_ref = torch.empty((M, N), dtype=torch.float16, device=DEV)
    h.gemm(x, y_ref, path)  # the existing entry point, with a caller workspace
    ref = y_ref.float().cpu().numpy()
    for _ in range(2):  # two calls in a row reuse the same scratch
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device=DEV)
        h.gemm_static(x, y, path)
        torch.cuda.synchronize()
        assert orc.rel_err(y.float().cpu().numpy(), ref) < tol
    assert h.device_error() == 0


def test_static_scratch_rejects_oversize_workspace():
    K, N, M = 5120, 256, 1024  # act-order gather alone needs M*K*2 = 10 MiB > 8 MiB
    layer = synthetic.make_layer(K, N, 128, act_order=True, seed=77)
    h = _handle(layer)
    assert h.workspace_size(M, torch.float16, _capi.PATH_AUTO) > (8 << 20)
    x = torch.zeros((M, K), dtype=torch.float16, device=DEV)
    y = torch.empty((M, N), dtype=torch.float16, device=DEV)
    with pytest.raises(_capi.W4A16Error) as ei:
        h.gemm_static(x, y)
    assert ei.value.code == _capi.W4A16_ERR_WORKSPACE
    assert "w4a16_gemm with a caller-provided workspace" in str(ei.value)


def test_static_scratch_checks_arguments_first():
    """A bad path or a null X is refused before any scratch look-up or size check."""
    layer = synthetic.make_layer(512, 256, 128, seed=78)
    h = _handle(layer)
    x = torch.zeros((1, 512), dtype=torch.float16, device=DEV)
    y = torch.empty((1, 256), dtype=torch.float16, device=DEV)
    with pytest.raises(_capi.W4A16Error) as ei:
        h.gemm_static(x, y, path=9)
    assert ei.value.code == _capi.W4A16_ERR_INVALID and "unknown path" in str(ei.value)
