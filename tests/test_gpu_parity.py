"""Parity of the CUDA path (through the C ABI) against the CPU oracle.

Dequant: bit-exact. GEMM/GEMV: max|Y - Y_ref| / max|Y_ref| <= 1e-2 (the north-star
tolerance; the observed error is far smaller and tighter bounds are asserted where
the arithmetic allows). Y_ref = X.float() @ W.float() from the oracle.
"""
import os

import numpy as np
import pytest
import torch

from drofell_for_revision_b200 import _capi, exllama, real_quant, synthetic
from oracle import w4a16_oracle as orc

pytestmark = pytest.mark.gpu

TOL = 1e-2
TOL_TC = 2e-3       # exact weights + fp32 accumulation: only the final rounding of Y remains
TOL_GEMV = 4e-3     # fp16 GEMV: half2 partials over at most 16 k, fp32 across them
DEV = torch.device("cuda:0")


def _handle(layer, device=DEV):
    return _capi.Handle(layer.qweight.to(device), layer.qzeros.to(device), layer.scales.to(device),
                        layer.g_idx if layer.act_order else None, device.index or 0)


def _ref(layer, x_cpu, dtype="fp16"):
    gi = layer.g_idx.numpy() if layer.act_order else None
    if dtype == "fp16":
        return orc.w4a16_linear_ref(x_cpu.numpy(), layer.qweight.numpy(), layer.qzeros.numpy(),
                                    layer.scales.numpy(), gi, layer.group_size)
    xb = x_cpu.view(torch.int16).numpy().view(np.uint16)
    return orc.w4a16_linear_ref(xb, layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(), gi,
                                layer.group_size, dtype="bf16")


def _gemm(h, x_cpu, path, dtype=torch.float16):
    x = x_cpu.to(DEV, dtype)
    y = torch.empty((x.shape[0], h.N), dtype=dtype, device=DEV)
    h.gemm(x, y, path)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


# ----------------------------------------------------------------------------- dequant
def test_dequant_golden_bit_exact(golden):
    for name, c in golden.items():
        layer = synthetic.GPTQLayer(torch.from_numpy(c["qweight"]), torch.from_numpy(c["qzeros"]),
                                    torch.from_numpy(c["scales"]), torch.from_numpy(c["g_idx"]),
                                    c["group_size"], c["act_order"])
        h = _handle(layer)
        w16 = torch.empty((c["K"], c["N"]), dtype=torch.float16, device=DEV)
        h.dequant(w16)
        wb = torch.empty((c["K"], c["N"]), dtype=torch.bfloat16, device=DEV)
        h.dequant(wb)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(w16.cpu().view(torch.int16).numpy().view(np.uint16),
                                      c["w_fp16"].view(np.uint16), err_msg=name)
        np.testing.assert_array_equal(wb.cpu().view(torch.int16).numpy().view(np.uint16), c["w_bf16_bits"],
                                      err_msg=name)


@pytest.mark.parametrize("K,N,g,act", [(4096, 4096, 128, False), (5120, 1024, 128, True), (1024, 96, 32, False),
                                       (11008, 256, 128, False), (256, 4096, -1, False)])
def test_dequant_synthetic_bit_exact(K, N, g, act):
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=K + N)
    h = _handle(layer)
    w16 = torch.empty((K, N), dtype=torch.float16, device=DEV)
    h.dequant(w16)
    torch.cuda.synchronize()
    ref = orc.dequant_fp16(layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(),
                           layer.g_idx.numpy() if act else None, layer.group_size)
    np.testing.assert_array_equal(w16.cpu().view(torch.int16).numpy().view(np.uint16), ref.view(np.uint16))


# ----------------------------------------------------------------------------- GEMV
GEMV_SHAPES = [(4096, 4096, 128, False), (4096, 1024, 128, True), (1024, 96, 32, False), (11008, 512, 128, False),
               (512, 11008, 64, True), (192, 64, 24, False), (256, 160, 16, False), (512, 256, -1, False)]


def _gemv_handle(layer, kernel):
    """Handle whose GEMV is the repacked-weight mma.sync kernel for every M
    (kernel="mma", when the group size allows it) or the CUDA-core kernel
    (kernel="cuda": no repacked copy)."""
    env = {"mma": ("W4A16_GEMV_MMA_MIN_M", "1"), "cuda": ("W4A16_NO_REPACK", "1")}[kernel]
    os.environ[env[0]] = env[1]
    try:
        return _handle(layer)
    finally:
        del os.environ[env[0]]


@pytest.mark.parametrize("kernel", ["mma", "cuda"])
@pytest.mark.parametrize("K,N,g,act", GEMV_SHAPES)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 9, 13, 16, 21])
def test_gemv_parity(K, N, g, act, M, kernel):
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=7 * K + N)
    x = synthetic.make_activations(M, K, seed=M)
    h = _gemv_handle(layer, kernel)
    kern = h.plan(M, torch.float16, _capi.PATH_GEMV)[0]
    gs = K if g == -1 else g
    assert kern == (_capi.KERN_GEMV_MMA if kernel == "mma" and gs % 16 == 0 else _capi.KERN_GEMV)
    y = _gemm(h, x, _capi.PATH_GEMV)
    err = orc.rel_err(y, _ref(layer, x))
    # mma.sync: exact products, fp32 accumulate; CUDA cores: fp16 partials over <= 16 k
    assert err < (TOL_TC if kern == _capi.KERN_GEMV_MMA else TOL_GEMV), err


@pytest.mark.parametrize("kernel", ["mma", "cuda"])
@pytest.mark.parametrize("K,N,g,act", GEMV_SHAPES)
@pytest.mark.parametrize("M", [1, 3, 8, 12])
def test_gemv_parity_bf16(K, N, g, act, M, kernel):
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=9 * K + N)
    x = synthetic.make_activations(M, K, seed=50 + M, dtype=torch.bfloat16)
    h = _gemv_handle(layer, kernel)
    y = _gemm(h, x, _capi.PATH_GEMV, torch.bfloat16)
    err = orc.rel_err(y, _ref(layer, x, "bf16"))
    assert err < TOL, err  # exact (q - z) times bf16 X, fp32 group sums


# Shapes for the mma.sync GEMV's work split: K = one group, one stripe over a cluster
# of up to 16 CTAs, CTAs of 1, 2 and 4 stripes, N not a multiple of 64 (a half stripe,
# a stripe past N in a 4-stripe CTA), 16-row groups, groups longer than 128 rows,
# full-K groups, act-order.
SPLIT_SHAPES = [(128, 8192, 128, False), (11008, 64, 128, False), (28672, 1024, 128, False),
                (4096, 22016, 128, False), (1024, 96, 16, False), (8192, 320, 256, False),
                (4096, 544, -1, False), (2048, 1056, 128, True), (2048, 12320, 128, False),
                (4096, 4128, 128, True)]


@pytest.mark.parametrize("K,N,g,act", SPLIT_SHAPES)
@pytest.mark.parametrize("M", [1, 2, 8, 16])
def test_gemv_mma_work_split(K, N, g, act, M):
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=K + 13 * N + M)
    h = _gemv_handle(layer, "mma")
    assert h.plan(M, torch.float16, _capi.PATH_GEMV)[0] == _capi.KERN_GEMV_MMA
    x = synthetic.make_activations(M, K, seed=400 + M).to(DEV)
    ys = []
    for _ in range(3):  # the stripe counters are back at zero after every launch
        y = torch.full((M, N), float("nan"), dtype=torch.float16, device=DEV)  # unwritten stays NaN
        h.gemm(x, y, _capi.PATH_GEMV)
        ys.append(y)
    torch.cuda.synchronize()
    assert all(torch.equal(ys[0], yy) for yy in ys[1:])  # fixed summation order
    assert orc.rel_err(ys[0].float().cpu().numpy(), _ref(layer, x.cpu())) < TOL_TC
    assert h.device_error() == 0


# ----------------------------------------------------------------------------- tcgen05 GEMM
@pytest.mark.parametrize("K,N,g,act", [(4096, 4096, 128, False), (1024, 1024, 128, True), (96, 96, 32, False),
                                       (2048, 384, 64, False), (1024, 11008, 128, False), (256, 128, 16, False),
                                       (192, 64, 24, False), (512, 256, -1, False), (11008, 256, 128, True)])
@pytest.mark.parametrize("M", [1, 7, 16, 17, 64, 100, 128, 129, 256, 300, 700])
def test_tc_parity_fp16(K, N, g, act, M):
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=3 * K + N + M)
    x = synthetic.make_activations(M, K, seed=100 + M)
    h = _handle(layer)
    y = _gemm(h, x, _capi.PATH_TC)
    err = orc.rel_err(y, _ref(layer, x))
    assert err < TOL_TC, err


@pytest.mark.parametrize("K,N,g,act", [(4096, 4096, 128, False), (1024, 1024, 128, True), (96, 96, 32, False),
                                       (192, 64, 24, False), (11008, 256, 128, True)])
@pytest.mark.parametrize("M", [1, 5, 16])
def test_tc_exact_parity_small_m(K, N, g, act, M):
    """The exact-W GEMM at decode sizes."""
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=11 * K + N + M)
    x = synthetic.make_activations(M, K, seed=300 + M)
    h = _handle(layer)
    assert h.plan(M, torch.float16, _capi.PATH_TC_EXACT)[0] == _capi.KERN_EXACT
    y = _gemm(h, x, _capi.PATH_TC_EXACT)
    assert orc.rel_err(y, _ref(layer, x)) < TOL_TC


def test_kernel_selection():
    layer = synthetic.make_layer(4096, 1024, 128, seed=12)
    h = _handle(layer)
    for M in (1, 8, 16):
        assert h.plan(M, torch.float16, _capi.PATH_TC)[0] == _capi.KERN_EXACT
    for M in (1, 2):
        assert h.plan(M, torch.float16, _capi.PATH_AUTO)[0] == _capi.KERN_GEMV
        assert h.plan(M, torch.bfloat16, _capi.PATH_AUTO)[0] == _capi.KERN_GEMV
    for M in (3, 8, 16):
        assert h.plan(M, torch.float16, _capi.PATH_AUTO)[0] == _capi.KERN_GEMV_MMA
        assert h.plan(M, torch.bfloat16, _capi.PATH_AUTO)[0] == _capi.KERN_GEMV_MMA
    assert h.plan(17, torch.float16, _capi.PATH_TC)[0] == _capi.KERN_EXACT
    assert h.plan(1, torch.bfloat16, _capi.PATH_TC)[0] == _capi.KERN_EXACT


@pytest.mark.parametrize("K,N,g,act", [(4096, 4096, 128, False), (1024, 512, 64, True)])
@pytest.mark.parametrize("M", [1, 33, 256, 520])
def test_tc_parity_bf16(K, N, g, act, M):
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=5 * K + N + M)
    x = synthetic.make_activations(M, K, seed=200 + M, dtype=torch.bfloat16)
    h = _handle(layer)
    y = _gemm(h, x, _capi.PATH_TC, torch.bfloat16)
    err = orc.rel_err(y, _ref(layer, x, "bf16"))
    assert err < 8e-3, err  # bf16 output rounding (2^-9) dominates


@pytest.mark.parametrize("path", [_capi.PATH_TC, _capi.PATH_TC_EXACT, _capi.PATH_GEMV])
def test_deterministic_split_k(path):
    layer = synthetic.make_layer(8192, 1024, 128, seed=9)
    h = _handle(layer)
    assert h.plan(4, torch.float16, path)[2] > 1  # K split engaged
    x = synthetic.make_activations(4, 8192, seed=1).to(DEV)
    y1 = torch.empty((4, 1024), dtype=torch.float16, device=DEV)
    y2 = torch.empty_like(y1)
    h.gemm(x, y1, path)
    h.gemm(x, y2, path)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert orc.rel_err(y1.float().cpu().numpy(), _ref(layer, x.cpu())) < TOL
    assert h.device_error() == 0


def test_golden_linear_through_both_paths(golden):
    for name, c in golden.items():
        if name.startswith("extreme") or "uneven" in name:
            continue
        layer = synthetic.GPTQLayer(torch.from_numpy(c["qweight"]), torch.from_numpy(c["qzeros"]),
                                    torch.from_numpy(c["scales"]), torch.from_numpy(c["g_idx"]),
                                    c["group_size"], c["act_order"])
        h = _handle(layer)
        x = torch.from_numpy(c["x_fp16"])
        for path in (_capi.PATH_GEMV, _capi.PATH_TC):
            y = _gemm(h, x, path)
            assert orc.rel_err(y, c["y_fp32"]) < TOL, (name, path)
        xb = torch.from_numpy(c["x_bf16_bits"].view(np.int16)).view(torch.bfloat16)
        y = _gemm(h, xb, _capi.PATH_TC, torch.bfloat16)
        assert orc.rel_err(y, c["y_bf16_fp32"]) < TOL, name


def test_uneven_groups_golden_through_operator(golden):
    """Act-order groups of unequal sizes (the golden case): the handle pads every group
    to the longest one, the kernels run, and the result matches the golden."""
    c = golden["act_uneven_g64_k256_n64"]
    layer = synthetic.GPTQLayer(torch.from_numpy(c["qweight"]), torch.from_numpy(c["qzeros"]),
                                torch.from_numpy(c["scales"]), torch.from_numpy(c["g_idx"]), c["group_size"], True)
    h = _handle(layer)
    x = torch.from_numpy(c["x_fp16"]).to(DEV)
    for path in (_capi.PATH_AUTO, _capi.PATH_GEMV, _capi.PATH_TC):
        y = torch.empty((x.shape[0], c["N"]), dtype=torch.float16, device=DEV)
        h.gemm(x, y, path)
        torch.cuda.synchronize()
        assert orc.rel_err(y.float().cpu().numpy(), c["y_fp32"]) < TOL, path
    ql = _quant_linear(layer)
    assert orc.rel_err(ql(x).float().cpu().numpy(), c["y_fp32"]) < TOL


def test_unaligned_groups_run_on_the_kernels():
    """Groups whose sizes are not multiples of 8 rows: padded inside the handle, so the
    GEMV and the GEMM both run; the dequant stays bit-exact for any g_idx."""
    K, N, g = 256, 64, 64
    layer = synthetic.make_layer(K, N, g, act_order=True, seed=81)
    sizes = [60, 68, 64, 64]
    gi = torch.cat([torch.full((n,), i, dtype=torch.int32) for i, n in enumerate(sizes)])
    gi = gi[torch.randperm(K, generator=torch.Generator().manual_seed(82))]
    layer = synthetic.GPTQLayer(layer.qweight, layer.qzeros, layer.scales, gi, g, True)
    h = _handle(layer)
    for M in (3, 40):
        x = synthetic.make_activations(M, K, seed=83 + M)
        y = torch.empty((M, N), dtype=torch.float16, device=DEV)
        h.gemm(x.to(DEV), y)
        torch.cuda.synchronize()
        assert orc.rel_err(y.float().cpu().numpy(), _ref(layer, x)) < TOL, M
    ql = _quant_linear(layer)
    x = synthetic.make_activations(3, K, seed=83)
    out = ql(x.to(DEV)).float().cpu().numpy()
    assert orc.rel_err(out, _ref(layer, x)) < TOL
    w = ql.get_reconstruct_weights()  # dequant stays bit-exact for any g_idx
    ref = orc.dequant_fp16(layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(), gi.numpy(), g)
    np.testing.assert_array_equal(w.cpu().view(torch.int16).numpy().view(np.uint16), ref.view(np.uint16))


# ----------------------------------------------------------------------------- operator level
def _quant_linear(layer, bias=None):
    ql = real_quant.QuantLinear(layer.group_size, layer.K, layer.N, bias is not None, layer.act_order)
    ql.qweight.copy_(layer.qweight); ql.qzeros.copy_(layer.qzeros); ql.scales.copy_(layer.scales)
    ql.g_idx.copy_(layer.g_idx)
    if bias is not None:
        ql.bias.copy_(bias)
    ql = ql.to(DEV)
    ql.post_init(exllama.TuningParams(), exllama.CacheV2(DEV))
    return ql


@pytest.mark.parametrize("act", [False, True])
@pytest.mark.parametrize("shape", [(1, 1), (2, 3), (4, 64), (1, 2048)])
def test_quantlinear_forward(act, shape):
    layer = synthetic.make_layer(1024, 768, 128, act_order=act, seed=31)
    bias = (torch.randn(768) * 0.1).half()
    ql = _quant_linear(layer, bias)
    x = synthetic.make_activations(shape[0] * shape[1], 1024, seed=32).view(*shape, 1024)
    y = ql(x.to(DEV))
    assert y.shape == (*shape, 768) and y.dtype == torch.float16
    ref = _ref(layer, x.view(-1, 1024)) + bias.float().numpy()[None, :]
    assert orc.rel_err(y.view(-1, 768).float().cpu().numpy(), ref) < TOL


def test_quantlinear_backward_input_grad():
    layer = synthetic.make_layer(512, 256, 64, act_order=True, seed=41)
    ql = _quant_linear(layer)
    x = synthetic.make_activations(8, 512, seed=42).to(DEV).requires_grad_(True)
    y = ql(x)
    gy = synthetic.make_activations(8, 256, seed=43).to(DEV)
    y.backward(gy)
    W = orc.dequant_fp16(layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(),
                         layer.g_idx.numpy(), layer.group_size).astype(np.float32)
    ref = gy.float().cpu().numpy() @ W.T
    assert orc.rel_err(x.grad.float().cpu().numpy(), ref) < TOL


def test_reconstructed_weight_path_and_getters():
    layer = synthetic.make_layer(512, 256, 128, seed=51)
    ql = _quant_linear(layer)
    w = ql.get_reconstruct_weights()
    ref = orc.dequant_fp16(layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(), None, 128)
    np.testing.assert_array_equal(w.cpu().view(torch.int16).numpy().view(np.uint16), ref.view(np.uint16))
    ql.q4_matrix.reconstruct_weight(torch.float16)
    x = synthetic.make_activations(3, 512, seed=52)
    y = ql(x.to(DEV)).float().cpu().numpy()
    assert orc.rel_err(y, _ref(layer, x)) < TOL
    ql.q4_matrix.release_weight()


def test_packed_tensors_not_mutated():
    layer = synthetic.make_layer(1024, 512, 128, act_order=True, seed=61)
    ql = _quant_linear(layer)
    x = synthetic.make_activations(130, 1024, seed=62).to(DEV)
    ql(x)
    ql(x[:1])
    torch.cuda.synchronize()
    assert torch.equal(ql.qweight.cpu(), layer.qweight)
    assert torch.equal(ql.qzeros.cpu(), layer.qzeros)
    assert torch.equal(ql.scales.cpu(), layer.scales)


def test_cuda_graph_capture_of_forward():
    layer = synthetic.make_layer(4096, 1024, 128, seed=71)
    ql = _quant_linear(layer)
    xs = {M: synthetic.make_activations(M, 4096, seed=72 + M).to(DEV) for M in (1, 16, 300)}
    ys = {}
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for M, x in xs.items():  # warm-up outside capture
            ql(x)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for M, x in xs.items():
            ys[M] = ql(x)
    g.replay()
    torch.cuda.synchronize()
    for M, x in xs.items():
        ref = _ref(layer, x.cpu())
        assert orc.rel_err(ys[M].float().cpu().numpy(), ref) < TOL, M


# ----------------------------------------------------------------------------- full benchmark sizes
def _column_subset_ref(layer, x_cpu, cols):
    """Oracle on 8-aligned column blocks only (cheap at full size)."""
    qw = layer.qweight[:, cols].numpy()
    blocks = sorted(set(int(c) // 8 for c in cols))
    qz = layer.qzeros[:, blocks].numpy()
    sc = layer.scales[:, cols].numpy()
    gi = layer.g_idx.numpy() if layer.act_order else None
    return orc.w4a16_linear_ref(x_cpu.numpy(), qw, qz, sc, gi, layer.group_size)


@pytest.mark.parametrize("K,N,act,M", [(4096, 11008, False, 1), (11008, 4096, False, 8), (4096, 11008, False, 2048),
                                       (5120, 13824, True, 1), (13824, 5120, True, 1024), (8192, 1024, False, 16)])
def test_full_size_properties(K, N, act, M):
    layer = synthetic.make_layer(K, N, 128, act_order=act, seed=K ^ N)
    h = _handle(layer)
    x = synthetic.make_activations(M, K, seed=M)
    xd = x.to(DEV)
    y = torch.empty((M, N), dtype=torch.float16, device=DEV)
    h.gemm(xd, y)
    # 1) 8-aligned column blocks against the oracle
    rng = np.random.default_rng(K + N)
    starts = rng.choice(N // 8, size=6, replace=False) * 8
    cols = np.concatenate([np.arange(s, s + 8) for s in sorted(starts)])
    ref = _column_subset_ref(layer, x, cols)
    assert orc.rel_err(y[:, cols].float().cpu().numpy(), ref) < TOL
    # 2) linearity in X
    x2 = synthetic.make_activations(M, K, seed=M + 1).to(DEV)
    y2 = torch.empty_like(y)
    y12 = torch.empty_like(y)
    h.gemm(x2, y2)
    h.gemm((xd.float() + x2.float()).half(), y12)
    assert orc.rel_err(y12.float().cpu().numpy(), (y.float() + y2.float()).cpu().numpy()) < TOL
    # 3) every path agrees with a torch fp32 GEMM on the bit-exact dequantized weight
    w = torch.empty((K, N), dtype=torch.float16, device=DEV)
    h.dequant(w)
    torch.backends.cuda.matmul.allow_tf32 = False
    yref = (xd.float() @ w.float()).cpu().numpy()
    assert orc.rel_err(y.float().cpu().numpy(), yref) < TOL
    if M <= 8:
        yg = torch.empty_like(y)
        h.gemm(xd, yg, _capi.PATH_GEMV)
        assert orc.rel_err(yg.float().cpu().numpy(), yref) < TOL
    yt = torch.empty_like(y)
    h.gemm(xd, yt, _capi.PATH_TC)
    assert orc.rel_err(yt.float().cpu().numpy(), yref) < TOL_TC
    torch.cuda.synchronize()
    assert h.device_error() == 0


def test_qzeros_off_16_byte_alignment_matches_aligned():
    # qzeros need only be 4-byte aligned; the tcgen05 GEMMs bulk-copy zero rows, so the
    # handle keeps its own aligned copy of such a buffer: every kernel family then gives
    # the same bits as for an aligned qzeros
    K, N = 2048, 2048
    layer = synthetic.make_layer(K, N, 128, seed=41)
    qz = layer.qzeros.to(DEV)
    buf = torch.empty(qz.numel() + 4, dtype=torch.int32, device=DEV)
    off = buf[1:1 + qz.numel()].view(qz.shape)  # 4 bytes past a 16-byte boundary
    off.copy_(qz)
    assert off.data_ptr() % 16 == 4
    qw, sc = layer.qweight.to(DEV), layer.scales.to(DEV)
    h0 = _capi.Handle(qw, qz, sc, None, 0)
    h1 = _capi.Handle(qw, off, sc, None, 0)
    for M in (1, 8, 64, 512):  # CUDA-core GEMV, mma.sync GEMV, natural-orientation and swap-AB GEMM
        x = synthetic.make_activations(M, K, seed=M).to(DEV)
        y0 = torch.empty((M, N), dtype=torch.float16, device=DEV)
        y1 = torch.full((M, N), float("nan"), dtype=torch.float16, device=DEV)
        h0.gemm(x, y0)
        h1.gemm(x, y1)
        torch.cuda.synchronize()
        assert torch.equal(y0, y1), M
    w0 = torch.empty((K, N), dtype=torch.float16, device=DEV)
    w1 = torch.empty_like(w0)
    h0.dequant(w0)
    h1.dequant(w1)
    assert torch.equal(w0, w1)
    assert h0.device_error() == 0 and h1.device_error() == 0
    h0.close()
    h1.close()
