"""The CPU oracle pinned against golden vectors produced by the reference's own code.

Goldens come from After-Revision-DROFELL/operators/core/linear/real_quant.py:69-102
(see tests/golden/make_golden.py). Dequant must match bit for bit.
"""
import numpy as np
import pytest

from oracle import w4a16_oracle as orc


def test_golden_cases_present(golden):
    assert len(golden) >= 9
    assert any(c["act_order"] for c in golden.values())


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_dequant_fp16_bit_exact(golden, impl):
    for name, c in golden.items():
        gi = c["g_idx"] if c["act_order"] else None
        if impl == "numpy":
            w = orc.dequant_fp16(c["qweight"], c["qzeros"], c["scales"], gi, c["group_size"])
        else:
            w = orc.c_dequant_fp16(c["qweight"], c["qzeros"], c["scales"], gi, c["group_size"], threads=2)
        assert w.dtype == np.float16
        np.testing.assert_array_equal(w.view(np.uint16), c["w_fp16"].view(np.uint16), err_msg=name)


def test_dequant_default_g_idx_equals_explicit(golden):
    for name, c in golden.items():
        if c["act_order"]:
            continue
        w1 = orc.dequant_fp16(c["qweight"], c["qzeros"], c["scales"], None, c["group_size"])
        w2 = orc.dequant_fp16(c["qweight"], c["qzeros"], c["scales"], c["g_idx"], c["group_size"])
        np.testing.assert_array_equal(w1.view(np.uint16), w2.view(np.uint16), err_msg=name)


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_dequant_bf16_bit_exact(golden, impl):
    for name, c in golden.items():
        gi = c["g_idx"] if c["act_order"] else None
        if impl == "numpy":
            w = orc.dequant_bf16_bits(c["qweight"], c["qzeros"], c["scales"], gi, c["group_size"])
        else:
            w = orc.c_dequant_bf16_bits(c["qweight"], c["qzeros"], c["scales"], gi, c["group_size"])
        np.testing.assert_array_equal(w, c["w_bf16_bits"], err_msg=name)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_linear_matches_golden(golden, dtype):
    for name, c in golden.items():
        if name.startswith("extreme"):
            continue  # infinities in W make the fp32 product non-finite; dequant is checked above
        gi = c["g_idx"] if c["act_order"] else None
        x = c["x_fp16"] if dtype == "fp16" else c["x_bf16_bits"]
        ref = c["y_fp32"] if dtype == "fp16" else c["y_bf16_fp32"]
        y_np = orc.w4a16_linear_ref(x, c["qweight"], c["qzeros"], c["scales"], gi, c["group_size"], dtype=dtype)
        y_c = orc.c_linear(x, c["qweight"], c["qzeros"], c["scales"], gi, c["group_size"], dtype=dtype, threads=2)
        assert orc.rel_err(y_np, ref) < 1e-5, name
        assert orc.rel_err(y_c, ref) < 1e-5, name


def test_known_answer_hand_built():
    # K=8, N=8, one group of 8: qweight row packs q[k, n] = (k + n) % 16, zero nibble n -> z = n + 1
    K, N = 8, 8
    q = np.array([[(k + n) % 16 for n in range(N)] for k in range(K)], dtype=np.int64)
    qweight = np.zeros((1, N), dtype=np.int64)
    for k in range(K):
        qweight[0] |= q[k] << (4 * k)
    qweight = qweight.astype(np.uint32).view(np.int32)
    qz = np.zeros((1, 1), dtype=np.int64)
    for n in range(N):
        qz[0, 0] |= n << (4 * n)
    qzeros = qz.astype(np.uint32).view(np.int32)
    scales = np.full((1, N), 0.5, dtype=np.float16)
    w = orc.dequant_fp16(qweight, qzeros, scales, group_size=8)
    expect = np.array([[0.5 * (((k + n) % 16) - (n + 1)) for n in range(N)] for k in range(K)], dtype=np.float16)
    np.testing.assert_array_equal(w, expect)


def test_rounding_is_single_rne():
    # scale 0.1 (fp16 0.0999755859375) * 3 = 0.29992675... -> RNE to fp16
    qweight = np.array([[3] * 8], dtype=np.int32)          # q[0, n] = 3, others 0
    qzeros = np.array([[(-1) & 0]], dtype=np.int32)       # z = 1 for all -> q - z = 2 / -1
    scales = np.full((1, 8), 0.1, dtype=np.float16)
    w = orc.dequant_fp16(qweight, qzeros, scales, group_size=8)
    s = np.float32(np.float16(0.1))
    assert w[0, 0] == np.float16(s * np.float32(2.0))
    assert w[1, 0] == np.float16(s * np.float32(-1.0))


def test_act_order_perm_is_stable_counting_sort():
    rng = np.random.default_rng(0)
    g_idx = rng.integers(0, 4, size=64).astype(np.int32)
    perm = orc.act_order_perm(g_idx, 4)
    np.testing.assert_array_equal(perm, np.argsort(g_idx, kind="stable"))


def test_rel_err_definition():
    assert orc.rel_err(np.array([1.0, 2.0]), np.array([1.0, 2.0])) == 0.0
    assert abs(orc.rel_err(np.array([1.0, 2.2]), np.array([1.0, 2.0])) - 0.1) < 1e-12


def test_rms_norm_and_silu_mul_restatements():
    """The oracle's RMSNorm and silu * mul against independent fp64 evaluations of the
    reference formulas (fuse_v2/rms_norm.cu:48-91, fuse_v2/q_mlp.cu:12-33,44-85)."""
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((3, 256)) * 4).astype(np.float16)
    w = (1 + 0.1 * rng.standard_normal(256)).astype(np.float16)
    eps = 1e-5
    xd = x.astype(np.float64)
    ref = xd * w.astype(np.float64) / np.sqrt((xd * xd).mean(axis=1, keepdims=True) + eps)
    got = orc.rms_norm_ref(x, w, eps).astype(np.float64)
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-3)) < 2e-3
    g = (rng.standard_normal((2, 64)) * 5).astype(np.float16)
    u = rng.standard_normal((2, 64)).astype(np.float16)
    gd = g.astype(np.float64)
    ref = gd / (1 + np.exp(-gd)) * u.astype(np.float64)
    got = orc.silu_mul_ref(g, u).astype(np.float64)
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-3)) < 2e-3
    # clamping to the fp16 range: an infinite input stays finite after the norm
    x2 = np.array([[np.inf, 1.0] + [0.0] * 6], dtype=np.float16)
    assert np.isfinite(orc.rms_norm_ref(x2, np.ones(8, np.float16), eps).astype(np.float32)).all()
