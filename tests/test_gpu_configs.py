"""Parity at the benchmark's own shapes (benchmark configs 2-5), through the C ABI.

Every case runs the kernel configuration the planner picks for the full-size shape
(the one the bench times) and compares against the CPU oracle:
  * the WIDE CUDA-core GEMV (merged qkv 4096x12288 and gate_up 4096x22016 at M=1,
    the bench's roofline kernel) on the whole output;
  * Llama-2-70B q/o, k/v, gate/up and down at M = 1, 16, 128, 2048, Llama-2-13B with
    act-order at M = 128 and Llama-2-7B at M = 512 on 8-aligned column blocks (the
    oracle over the full weight would take minutes), plus the whole output against a
    torch fp32 GEMM on the bit-exact dequantized weight.
Tolerance: max|Y - Y_ref| / max|Y_ref| <= 1e-2, with the
kernels' tighter bounds where the arithmetic allows.
"""
import os

import numpy as np
import pytest
import torch

from drofell_for_revision_b200 import _capi, synthetic
from oracle import w4a16_oracle as orc

pytestmark = pytest.mark.gpu

TOL = 1e-2
TOL_TC = 2e-3
TOL_GEMV = 4e-3
DEV = torch.device("cuda:0")

_LAYERS = {}


def _layer(K, N, act=False):
    key = (K, N, act)
    if key not in _LAYERS:
        _LAYERS.clear()  # one full-size layer resident at a time (host memory)
        _LAYERS[key] = synthetic.make_layer(K, N, 128, act_order=act, seed=(K * 31 + N) ^ (7 if act else 0))
    return _LAYERS[key]


def _handle(layer):
    return _capi.Handle(layer.qweight.to(DEV), layer.qzeros.to(DEV), layer.scales.to(DEV),
                        layer.g_idx if layer.act_order else None, 0)


def _cols(N, seed, blocks=8):
    rng = np.random.default_rng(seed)
    starts = np.sort(rng.choice(N // 8, size=min(blocks, N // 8), replace=False)) * 8
    starts[0] = 0                    # first and last column blocks always included
    starts[-1] = N - 8
    return np.unique(np.concatenate([np.arange(s, s + 8) for s in starts]))


def _subset_ref(layer, x_cpu, cols, dtype="fp16"):
    qw = layer.qweight[:, cols].numpy()
    qz = layer.qzeros[:, sorted(set(int(c) // 8 for c in cols))].numpy()
    sc = layer.scales[:, cols].numpy()
    gi = layer.g_idx.numpy() if layer.act_order else None
    if dtype == "bf16":
        xb = x_cpu.view(torch.int16).numpy().view(np.uint16)
        return orc.c_linear(xb, qw, qz, sc, gi, layer.group_size, dtype="bf16", threads=8)
    return orc.c_linear(x_cpu.numpy(), qw, qz, sc, gi, layer.group_size, threads=8)


# ----------------------------------------------------------------------------- WIDE GEMV
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("K,N", [(4096, 12288), (4096, 22016)])
def test_wide_gemv_full_output(K, N, dtype):
    """The merged qkv / gate_up projections at M = 1 run the WIDE CUDA-core GEMV
    (3 CTAs per SM, 4-row batches): the configuration behind the bench's value and
    roofline. Whole output against the oracle."""
    plan, wide, _ = _capi.plan_shape(K, N, K // 128, 1, dtype, _capi.PATH_AUTO, torch.cuda.get_device_properties(0).multi_processor_count)
    assert plan[0] == _capi.KERN_GEMV and wide, (plan, wide)
    layer = _layer(K, N)
    h = _handle(layer)
    assert h.plan(1, dtype) == plan
    x = synthetic.make_activations(1, K, seed=K + N, dtype=dtype)
    y = torch.full((1, N), float("nan"), dtype=dtype, device=DEV)
    h.gemm(x.to(DEV), y)
    torch.cuda.synchronize()
    dt = "bf16" if dtype == torch.bfloat16 else "fp16"
    xin = x.view(torch.int16).numpy().view(np.uint16) if dt == "bf16" else x.numpy()
    ref = orc.c_linear(xin, layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(), None, 128,
                       dtype=dt, threads=8)
    err = orc.rel_err(y.float().cpu().numpy(), ref)
    assert err < (TOL_GEMV if dt == "fp16" else TOL), err
    assert h.device_error() == 0


# ----------------------------------------------------------------------------- full configs
CONFIGS = (
    # Llama-2-70B (config 5): q/o, k/v, gate/up, down at M = 1, 16, 128, 2048
    [(8192, 8192, False, M) for M in (1, 16, 128, 2048)]
    + [(8192, 1024, False, M) for M in (1, 16, 128, 2048)]
    + [(8192, 28672, False, M) for M in (1, 16, 128, 2048)]
    + [(28672, 8192, False, M) for M in (1, 16, 128, 2048)]
    # Llama-2-13B with act-order (config 4) at M = 128, and its merged gate_up at M = 1
    # (the mma.sync GEMV over the group-sorted weight)
    + [(5120, 13824, True, 128), (13824, 5120, True, 128), (5120, 5120, True, 128), (5120, 27648, True, 1)]
    # Llama-2-7B (config 3) at M = 512
    + [(4096, 4096, False, 512), (4096, 11008, False, 512), (11008, 4096, False, 512)]
)


@pytest.mark.parametrize("K,N,act,M", CONFIGS)
def test_baseline_config(K, N, act, M):
    layer = _layer(K, N, act)
    h = _handle(layer)
    x = synthetic.make_activations(M, K, seed=M * 3 + K)
    xd = x.to(DEV)
    y = torch.full((M, N), float("nan"), dtype=torch.float16, device=DEV)
    h.gemm(xd, y)  # PATH_AUTO: the kernel the bench runs at this M
    torch.cuda.synchronize()
    kern = h.plan(M)[0]
    # 1) column blocks (first, last and random) against the oracle
    cols = _cols(N, K + N + M)
    ref = _subset_ref(layer, x, cols)
    tol = TOL_GEMV if kern == _capi.KERN_GEMV else TOL_TC
    assert orc.rel_err(y[:, cols].float().cpu().numpy(), ref) < tol
    # 2) the whole output against torch fp32 on the bit-exact dequantized weight
    w = torch.empty((K, N), dtype=torch.float16, device=DEV)
    h.dequant(w)
    torch.backends.cuda.matmul.allow_tf32 = False
    yref = xd.float() @ w.float()
    del w
    assert not torch.isnan(y).any()
    assert orc.rel_err(y.float().cpu().numpy(), yref.cpu().numpy()) < tol
    assert h.device_error() == 0


def test_70b_gate_m1_bf16_runs_the_mma_gemv():
    """70B gate at M = 1 runs the mma.sync GEMV (K >= 8192 and N >= 8192 stream faster
    there than on the CUDA-core kernel); bf16 against the oracle on column blocks, and
    against the CUDA-core kernel of a handle without the repacked copy."""
    K, N = 8192, 28672
    plan, _, _ = _capi.plan_shape(K, N, K // 128, 1, torch.bfloat16, _capi.PATH_AUTO, 148)
    assert plan[0] == _capi.KERN_GEMV_MMA
    layer = _layer(K, N)
    h = _handle(layer)
    x = synthetic.make_activations(1, K, seed=11, dtype=torch.bfloat16)
    y = torch.empty((1, N), dtype=torch.bfloat16, device=DEV)
    h.gemm(x.to(DEV), y)
    torch.cuda.synchronize()
    cols = _cols(N, 5)
    ref = _subset_ref(layer, x, cols, "bf16")
    assert orc.rel_err(y[:, cols].float().cpu().numpy(), ref) < TOL
    os.environ["W4A16_NO_REPACK"] = "1"
    try:
        hc = _handle(layer)
    finally:
        del os.environ["W4A16_NO_REPACK"]
    assert hc.plan(1, torch.bfloat16, _capi.PATH_AUTO)[0] == _capi.KERN_GEMV
    yc = torch.empty_like(y)
    hc.gemm(x.to(DEV), yc)
    torch.cuda.synchronize()
    assert orc.rel_err(y.float().cpu().numpy(), yc.float().cpu().numpy()) < TOL
    assert h.device_error() == 0 and hc.device_error() == 0
