"""The transposed W4A16 GEMM (w4a16_gemm_t: dX = dY W^T, the input gradient) against
the oracle, through the C ABI and through autograd.

Reference semantics: the backward of After-Revision-DROFELL/cuda_extends/exllama.py:
670-696 -> q4_transpose_matmul.cu:115-167 multiplies dY by the transpose of the
dense weight real_quant.py:69-90 defines. Y_ref = dY.float() @ W.float().T with W the
oracle's bit-exact dequant. Tolerance: max|dX - ref| / max|ref| <= 2e-3 (exact
weights, fp32 accumulation; only the final rounding of dX remains), 8e-3 for bf16
outputs, and the north-star 1e-2 at the operator level.
"""
import numpy as np
import pytest
import torch

from drofell_for_revision_b200 import _capi, exllama, real_quant, synthetic
from oracle import w4a16_oracle as orc

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
TOL_TC = 2e-3
TOL_BF16 = 8e-3


def _handle(layer):
    return _capi.Handle(layer.qweight.to(DEV), layer.qzeros.to(DEV), layer.scales.to(DEV),
                        layer.g_idx if layer.act_order else None, 0)


def _w_ref(layer, dtype="fp16"):
    gi = layer.g_idx.numpy() if layer.act_order else None
    if dtype == "bf16":
        return orc.bf16_bits_to_fp32(orc.c_dequant_bf16_bits(layer.qweight.numpy(), layer.qzeros.numpy(),
                                                             layer.scales.numpy(), gi, layer.group_size, threads=8))
    return orc.c_dequant_fp16(layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(), gi,
                              layer.group_size, threads=8).astype(np.float32)


def _dy(M, N, seed, dtype=torch.float16):
    return synthetic.make_activations(M, N, seed=seed, dtype=dtype)


@pytest.mark.parametrize("K,N,g,act", [(256, 128, 128, False), (1024, 768, 64, False), (512, 256, 32, True),
                                       (96, 96, 32, False), (4096, 1024, 128, True), (2048, 384, -1, False),
                                       (192, 64, 24, False), (1024, 96, 16, False)])
@pytest.mark.parametrize("M", [1, 7, 16, 64, 130, 300, 600])
def test_gemm_t_parity_fp16(K, N, g, act, M):
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=K + 7 * N + M)
    h = _handle(layer)
    dy = _dy(M, N, seed=M + 3)
    dx = torch.full((M, K), float("nan"), dtype=torch.float16, device=DEV)
    h.gemm_t(dy.to(DEV), dx)
    torch.cuda.synchronize()
    ref = dy.float().numpy() @ _w_ref(layer).T
    assert orc.rel_err(dx.float().cpu().numpy(), ref) < TOL_TC
    assert h.device_error() == 0


@pytest.mark.parametrize("K,N,g,act", [(1024, 512, 128, False), (512, 1024, 64, True)])
@pytest.mark.parametrize("M", [1, 33, 256, 520])
def test_gemm_t_parity_bf16(K, N, g, act, M):
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=3 * K + N + M)
    h = _handle(layer)
    dy = _dy(M, N, seed=M + 5, dtype=torch.bfloat16)
    dx = torch.empty((M, K), dtype=torch.bfloat16, device=DEV)
    h.gemm_t(dy.to(DEV), dx)
    torch.cuda.synchronize()
    ref = dy.float().numpy() @ _w_ref(layer, "bf16").T
    assert orc.rel_err(dx.float().cpu().numpy(), ref) < TOL_BF16


def _row_blocks(K, seed, blocks=8):
    rng = np.random.default_rng(seed)
    starts = np.sort(rng.choice(K // 8, size=min(blocks, K // 8), replace=False)) * 8
    starts[0], starts[-1] = 0, K - 8
    return np.unique(np.concatenate([np.arange(s, s + 8) for s in starts]))


# Llama-2-7B / 13B projections (the shapes a PEFT backward sees) at M = 1, 128, 2048
@pytest.mark.parametrize("K,N,act", [(4096, 4096, False), (4096, 11008, False), (11008, 4096, False),
                                     (5120, 13824, True), (13824, 5120, True)])
@pytest.mark.parametrize("M", [1, 128, 2048])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gemm_t_llama_shapes(K, N, act, M, dtype):
    layer = synthetic.make_layer(K, N, 128, act_order=act, seed=K ^ N ^ M)
    h = _handle(layer)
    dy = _dy(M, N, seed=M, dtype=dtype)
    dyd = dy.to(DEV)
    dx = torch.full((M, K), float("nan"), dtype=dtype, device=DEV)
    h.gemm_t(dyd, dx)
    torch.cuda.synchronize()
    dt = "bf16" if dtype == torch.bfloat16 else "fp16"
    tol = TOL_BF16 if dt == "bf16" else TOL_TC
    # 1) rows of W (columns of dX) against the oracle
    rows = _row_blocks(K, K + N + M)
    w = _w_ref(layer, dt)
    ref = dy.float().numpy() @ w[rows].T
    assert orc.rel_err(dx[:, rows].float().cpu().numpy(), ref) < tol
    # 2) the whole dX against torch fp32 on the bit-exact dequantized weight
    wd = torch.empty((K, N), dtype=dtype, device=DEV)
    h.dequant(wd)
    torch.backends.cuda.matmul.allow_tf32 = False
    full = dyd.float() @ wd.float().t()
    assert not torch.isnan(dx).any()
    assert orc.rel_err(dx.float().cpu().numpy(), full.cpu().numpy()) < tol
    assert h.device_error() == 0


def test_gemm_t_split_k_is_deterministic():
    layer = synthetic.make_layer(1024, 8192, 128, seed=4)
    h = _handle(layer)
    dy = _dy(64, 8192, seed=1).to(DEV)
    assert h.workspace_size_t(64, torch.float16) > 0  # few k tiles: the reduction over N is split
    a = torch.empty((64, 1024), dtype=torch.float16, device=DEV)
    b = torch.empty_like(a)
    h.gemm_t(dy, a)
    h.gemm_t(dy, b)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    ref = dy.float().cpu().numpy() @ _w_ref(layer).T
    assert orc.rel_err(a.float().cpu().numpy(), ref) < TOL_TC


def test_unequal_act_order_groups_run_on_the_kernels():
    """Act-order tables whose groups differ in size (padded to the longest group inside
    the handle): forward and transposed products on the kernels, no fallback."""
    K, N, g = 512, 256, 64
    base = synthetic.make_layer(K, N, g, act_order=True, seed=81)
    sizes = [40, 88, 64, 64, 70, 58, 64, 64]
    gi = torch.cat([torch.full((n,), i, dtype=torch.int32) for i, n in enumerate(sizes)])
    gi = gi[torch.randperm(K, generator=torch.Generator().manual_seed(82))]
    layer = synthetic.GPTQLayer(base.qweight, base.qzeros, base.scales, gi, g, True)
    h = _handle(layer)
    w = _w_ref(layer)
    for M in (1, 5, 40, 300):
        x = synthetic.make_activations(M, K, seed=M)
        y = torch.empty((M, N), dtype=torch.float16, device=DEV)
        h.gemm(x.to(DEV), y)
        dy = _dy(M, N, seed=M + 1)
        dx = torch.empty((M, K), dtype=torch.float16, device=DEV)
        h.gemm_t(dy.to(DEV), dx)
        torch.cuda.synchronize()
        assert orc.rel_err(y.float().cpu().numpy(), x.float().numpy() @ w) < 4e-3, M
        assert orc.rel_err(dx.float().cpu().numpy(), dy.float().numpy() @ w.T) < TOL_TC, M


@pytest.mark.parametrize("act", [False, True])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_quantlinear_backward_runs_the_transposed_kernel(act, dtype):
    K, N = 1024, 768
    layer = synthetic.make_layer(K, N, 128, act_order=act, seed=91)
    ql = real_quant.QuantLinear(128, K, N, False, act)
    ql.qweight.copy_(layer.qweight); ql.qzeros.copy_(layer.qzeros); ql.scales.copy_(layer.scales)
    ql.g_idx.copy_(layer.g_idx)
    ql = ql.to(DEV)
    ql.post_init(exllama.TuningParams(), exllama.CacheV2(DEV))
    x = synthetic.make_activations(2 * 37, K, seed=92, dtype=dtype).view(2, 37, K).to(DEV).requires_grad_(True)
    y = ql(x)
    gy = synthetic.make_activations(2 * 37, N, seed=93, dtype=dtype).view(2, 37, N).to(DEV)
    y.backward(gy)
    w = _w_ref(layer, "bf16" if dtype == torch.bfloat16 else "fp16")
    ref = gy.float().cpu().numpy().reshape(-1, N) @ w.T
    assert x.grad.shape == x.shape and x.grad.dtype == dtype
    assert orc.rel_err(x.grad.float().cpu().numpy().reshape(-1, K), ref) < 1e-2


def test_kernels_from_a_thread_that_never_used_cuda():
    """Driver entry points (the TMA descriptor encode) need the device's context current
    in the calling thread; a fresh worker thread, such as autograd's backward thread,
    has none until the library binds it. Forward GEMM, transposed GEMM and GEMV from a
    new thread must match the same calls on the main thread."""
    import threading
    layer = synthetic.make_layer(1024, 768, 128, seed=17)
    h = _handle(layer)
    x = synthetic.make_activations(74, 1024, seed=18).to(DEV)
    dy = _dy(74, 768, seed=19).to(DEV)

    def run():
        y = torch.empty((74, 768), dtype=torch.float16, device=DEV)
        y1 = torch.empty((1, 768), dtype=torch.float16, device=DEV)
        dx = torch.empty((74, 1024), dtype=torch.float16, device=DEV)
        h.gemm(x, y, _capi.PATH_TC)
        h.gemm(x[:1], y1)
        h.gemm_t(dy, dx)
        torch.cuda.synchronize()
        return y, y1, dx

    out, err = {}, []

    def worker():
        try:
            out["thread"] = run()
        except Exception as e:  # reported on the main thread
            err.append(e)

    t = threading.Thread(target=worker)
    t.start()
    t.join()
    assert not err, err
    ref = run()
    for a, b in zip(out["thread"], ref):
        assert torch.equal(a, b)
