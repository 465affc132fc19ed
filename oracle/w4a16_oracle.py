"""CPU restatement of the reference's GPTQ W4A16 dequantize-then-matmul semantics.

TEST INFRASTRUCTURE ONLY: this module is the checker for the CUDA path and the
timed CPU baseline. The product package never imports it.

Parity status: PINNED. ``tests/golden/make_golden.py`` runs the reference's own
``QuantLinear.get_reconstruct_weights`` (After-Revision-DROFELL/operators/core/
linear/real_quant.py:69-102) with the missing CUDA extension stubbed out and the
AutoGPTQ shift table ``wf = arange(0, 32, 4)`` supplied; the fixtures it writes
are compared bit-for-bit against :func:`dequant_fp16` by ``tests/test_oracle.py``.

Layout (After-Revision-DROFELL/operators/core/linear/real_quant.py:25-49):
  qweight int32 [K/8, N]   nibble i of qweight[r, n] is q[8r + i, n]
  qzeros  int32 [G, N/8]   nibble j of qzeros[g, c] is z_raw[g, 8c + j]
  scales  fp16  [G, N]
  g_idx   int32 [K]        group of input row k (default k // group_size)

Semantics (real_quant.py:69-90):
  z[g, n] = z_raw[g, n] + 1                      ("+1" GPTQ zero convention)
  W[k, n] = fp16( scales[g_idx[k], n] * (q[k, n] - z[g_idx[k], n]) )
The product of an fp16 scale and an integer in [-16, 14] is exact in fp32, so a
single round-to-nearest-even to fp16 reproduces torch's fp16 multiply exactly.

bf16 weights follow the reference's bf16 reconstruct kernel
(After-Revision-DROFELL/cuda_extends/exllama/q4_matrix.cu:465-467,569-579): the
fp16 weight is computed first and then converted fp16 -> fp32 -> bf16 (RNE).

GEMM semantics: Y = X.float() @ W.float() in fp32 (the north-star tolerance is
max|Y - Y_ref| / max|Y_ref| <= 1e-2).
"""
from __future__ import annotations

import numpy as np

SHIFTS = np.arange(0, 32, 4, dtype=np.int32)  # the ``wf`` table real_quant.py:72,81 shifts by


def unpack_qweight(qweight: np.ndarray) -> np.ndarray:
    """q[k, n] in 0..15 from qweight [K/8, N] (real_quant.py:79-86)."""
    qw = np.asarray(qweight, dtype=np.int32)
    kw, n = qw.shape
    w = (qw[:, None, :] >> SHIFTS[None, :, None]) & 15
    return w.reshape(kw * 8, n).astype(np.int8)


def unpack_qzeros(qzeros: np.ndarray) -> np.ndarray:
    """z[g, n] = nibble + 1 from qzeros [G, N/8] (real_quant.py:70-77)."""
    qz = np.asarray(qzeros, dtype=np.int32)
    g, c = qz.shape
    z = (qz[:, :, None] >> SHIFTS[None, None, :]) & 15
    return (z + 1).reshape(g, c * 8).astype(np.int8)


def default_g_idx(k: int, group_size: int) -> np.ndarray:
    """The default group table of real_quant.py:44-48: g_idx[k] = k // group_size."""
    return (np.arange(k, dtype=np.int64) // group_size).astype(np.int32)


def dequant_fp16(qweight, qzeros, scales, g_idx=None, group_size: int | None = None) -> np.ndarray:
    """W [K, N] fp16, bit-identical to real_quant.py:89-90 for num_itr == 1."""
    q = unpack_qweight(qweight)
    z = unpack_qzeros(qzeros)
    s = np.asarray(scales, dtype=np.float16)
    k = q.shape[0]
    if g_idx is None:
        if group_size is None:
            group_size = k // s.shape[0]
        g_idx = default_g_idx(k, group_size)
    gi = np.asarray(g_idx, dtype=np.int64)
    diff = (q.astype(np.int32) - z[gi].astype(np.int32)).astype(np.float32)
    prod = s[gi].astype(np.float32) * diff  # exact in fp32
    with np.errstate(over="ignore"):
        return prod.astype(np.float16)      # one RNE rounding, as torch's fp16 mul (overflow -> inf)


def fp32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (round to nearest even), returned as uint16 bit patterns."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_bits_to_fp32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def dequant_bf16_bits(qweight, qzeros, scales, g_idx=None, group_size: int | None = None) -> np.ndarray:
    """bf16 W as uint16 bits: bf16(fp32(fp16 W)), as q4_matrix.cu:465-467 converts."""
    w16 = dequant_fp16(qweight, qzeros, scales, g_idx, group_size)
    return fp32_to_bf16_bits(w16.astype(np.float32))


def matmul_fp32(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Y = X.float() @ W.float() (fp32 accumulate)."""
    return np.asarray(x, dtype=np.float32) @ np.asarray(w, dtype=np.float32)


def w4a16_linear_ref(x, qweight, qzeros, scales, g_idx=None, group_size=None, bias=None,
                     dtype: str = "fp16") -> np.ndarray:
    """Reference forward in fp32: dequant (fp16, or bf16 for bf16 activations) then fp32 matmul.

    ``x`` is an fp16 array, or a uint16 array of bf16 bits when ``dtype == 'bf16'``.
    """
    if dtype == "fp16":
        w = dequant_fp16(qweight, qzeros, scales, g_idx, group_size).astype(np.float32)
        xf = np.asarray(x, dtype=np.float16).astype(np.float32)
    elif dtype == "bf16":
        w = bf16_bits_to_fp32(dequant_bf16_bits(qweight, qzeros, scales, g_idx, group_size))
        xf = bf16_bits_to_fp32(x)
    else:
        raise ValueError(dtype)
    y = xf @ w
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)[None, :]
    return y


def act_order_perm(g_idx: np.ndarray, groups: int) -> np.ndarray:
    """Stable counting sort of rows by group: x_map of q4_matrix.cu:125-176.

    Returns ``perm`` with ``perm[j]`` = original row placed at sorted position j.
    """
    gi = np.asarray(g_idx, dtype=np.int64)
    counts = np.bincount(gi, minlength=groups)
    start = np.concatenate([[0], np.cumsum(counts)[:-1]])
    nxt = start.copy()
    inv = np.empty(gi.shape[0], dtype=np.int64)
    for row, grp in enumerate(gi):
        inv[row] = nxt[grp]
        nxt[grp] += 1
    perm = np.empty_like(inv)
    perm[inv] = np.arange(gi.shape[0])
    return perm.astype(np.int32)


def rel_err(y: np.ndarray, y_ref: np.ndarray) -> float:
    """max|Y - Y_ref| / max|Y_ref|, the north-star GEMM error measure."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    denom = float(np.max(np.abs(y_ref))) if y_ref.size else 1.0
    if denom == 0.0:
        denom = 1.0
    return float(np.max(np.abs(y - y_ref))) / denom if y.size else 0.0


# ---------------------------------------------------------------------------
# ctypes binding of the plain-C restatement (oracle/w4a16_oracle.c)
# ---------------------------------------------------------------------------
import ctypes
import os

_C = None


def c_oracle():
    """Load oracle/libw4a16_oracle.so (built by oracle/Makefile)."""
    global _C
    if _C is None:
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libw4a16_oracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"C oracle not built: {path} (run `make -C oracle`)")
        lib = ctypes.CDLL(path)
        P = ctypes.c_void_p
        I = ctypes.c_int
        lib.oracle_dequant_fp16.argtypes = [P, P, P, P, I, I, I, P, I]
        lib.oracle_dequant_fp16.restype = I
        lib.oracle_dequant_bf16.argtypes = [P, P, P, P, I, I, I, P, I]
        lib.oracle_dequant_bf16.restype = I
        lib.oracle_matmul_f16w.argtypes = [P, I, P, I, I, P, I, I]
        lib.oracle_matmul_f16w.restype = I
        lib.oracle_linear.argtypes = [P, I, P, P, P, P, I, I, I, P, P, I, I]
        lib.oracle_linear.restype = I
        _C = lib
    return _C


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def c_matmul_f16w(x, w, dtype: str = "fp16", threads: int = 1, out: np.ndarray | None = None) -> np.ndarray:
    """Y = X.float() @ W.float() in plain C (OpenMP over ``threads``): x [M, K] and w [K, N]
    as fp16 arrays, or uint16 bf16 bit patterns with ``dtype == 'bf16'``."""
    xa = np.ascontiguousarray(x)
    wa = np.ascontiguousarray(w)
    m, k = xa.shape
    n = wa.shape[1]
    y = out if out is not None else np.empty((m, n), dtype=np.float32)
    rc = c_oracle().oracle_matmul_f16w(_ptr(xa), m, _ptr(wa), k, n, _ptr(y), 1 if dtype == "bf16" else 0, threads)
    if rc != 0:
        raise RuntimeError(f"oracle_matmul_f16w rc={rc}")
    return y


def c_dequant_fp16(qweight, qzeros, scales, g_idx=None, group_size=None, threads: int = 1,
                   out: np.ndarray | None = None) -> np.ndarray:
    qw = np.ascontiguousarray(qweight, dtype=np.int32)
    qz = np.ascontiguousarray(qzeros, dtype=np.int32)
    sc = np.ascontiguousarray(scales, dtype=np.float16)
    k, n = qw.shape[0] * 8, qw.shape[1]
    g = sc.shape[0]
    if group_size is None:
        group_size = k // g
    gi = None if g_idx is None else np.ascontiguousarray(g_idx, dtype=np.int32)
    if out is None:
        out = np.empty((k, n), dtype=np.float16)
    rc = c_oracle().oracle_dequant_fp16(_ptr(qw), _ptr(qz), _ptr(sc), None if gi is None else _ptr(gi),
                                         k, n, group_size, _ptr(out), threads)
    if rc != 0:
        raise RuntimeError(f"oracle_dequant_fp16 rc={rc}")
    return out


def c_dequant_bf16_bits(qweight, qzeros, scales, g_idx=None, group_size=None, threads: int = 1) -> np.ndarray:
    qw = np.ascontiguousarray(qweight, dtype=np.int32)
    qz = np.ascontiguousarray(qzeros, dtype=np.int32)
    sc = np.ascontiguousarray(scales, dtype=np.float16)
    k, n = qw.shape[0] * 8, qw.shape[1]
    g = sc.shape[0]
    if group_size is None:
        group_size = k // g
    gi = None if g_idx is None else np.ascontiguousarray(g_idx, dtype=np.int32)
    out = np.empty((k, n), dtype=np.uint16)
    rc = c_oracle().oracle_dequant_bf16(_ptr(qw), _ptr(qz), _ptr(sc), None if gi is None else _ptr(gi),
                                         k, n, group_size, _ptr(out), threads)
    if rc != 0:
        raise RuntimeError(f"oracle_dequant_bf16 rc={rc}")
    return out


def c_linear(x, qweight, qzeros, scales, g_idx=None, group_size=None, dtype: str = "fp16",
             threads: int = 1, w_scratch: np.ndarray | None = None) -> np.ndarray:
    """Dequant + fp32 matmul in plain C (OpenMP over ``threads``). Returns fp32 Y [M, N]."""
    qw = np.ascontiguousarray(qweight, dtype=np.int32)
    qz = np.ascontiguousarray(qzeros, dtype=np.int32)
    sc = np.ascontiguousarray(scales, dtype=np.float16)
    k, n = qw.shape[0] * 8, qw.shape[1]
    g = sc.shape[0]
    if group_size is None:
        group_size = k // g
    gi = None if g_idx is None else np.ascontiguousarray(g_idx, dtype=np.int32)
    xa = np.ascontiguousarray(x)
    if xa.dtype not in (np.float16, np.uint16):
        raise TypeError("x must be fp16 or bf16 bits (uint16)")
    m = xa.shape[0]
    if w_scratch is None or w_scratch.size < k * n:
        w_scratch = np.empty(k * n, dtype=np.uint16)
    y = np.empty((m, n), dtype=np.float32)
    rc = c_oracle().oracle_linear(_ptr(xa), m, _ptr(qw), _ptr(qz), _ptr(sc),
                                  None if gi is None else _ptr(gi), k, n, group_size,
                                  _ptr(w_scratch), _ptr(y), 1 if dtype == "bf16" else 0, threads)
    if rc != 0:
        raise RuntimeError(f"oracle_linear rc={rc}")
    return y


# ---------------------------------------------------------------------------
# Decoder-layer blocks around the projections (the reference's fused decode path)
# ---------------------------------------------------------------------------
def rms_norm_ref(x, w, eps: float) -> np.ndarray:
    """fp16 RMSNorm of each row (After-Revision-DROFELL/cuda_extends/exllama/fuse_v2/
    rms_norm.cu:48-91): x clamped to the fp16 range, rmf = rsqrt(sum(x^2) / K + eps) in
    fp32, y = fp16(x * w * rmf)."""
    xf = np.clip(np.asarray(x, dtype=np.float16).astype(np.float32), -65504.0, 65504.0)
    k = xf.shape[1]
    ss = np.sum(xf * xf, axis=1, dtype=np.float32)
    rmf = (np.float32(1.0) / np.sqrt(ss * np.float32(1.0 / k) + np.float32(eps))).astype(np.float32)
    wf = np.asarray(w, dtype=np.float16).astype(np.float32)
    return ((xf * wf[None, :]) * rmf[:, None]).astype(np.float16)


def silu_mul_ref(gate, up) -> np.ndarray:
    """fp16(silu(gate) * up), silu(g) = g / (1 + e^-g) (fuse_v2/q_mlp.cu:12-33,44-85),
    evaluated in fp32 and rounded once."""
    g = np.asarray(gate, dtype=np.float16).astype(np.float32)
    u = np.asarray(up, dtype=np.float16).astype(np.float32)
    with np.errstate(over="ignore"):
        return (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float16)


def _proj_fp16(x, p) -> np.ndarray:
    """A projection as the fused blocks chain them: fp32 product rounded to the fp16 the
    kernels store. ``p`` = (qweight, qzeros, scales, g_idx or None, group_size)."""
    return w4a16_linear_ref(x, *p).astype(np.float16)


def mlp_ref(x, norm_w, eps: float, gate, up, down) -> np.ndarray:
    """The MLP block mlp_forward (fuse_v2/q_mlp.cu:96-133): RMSNorm, gate and up, silu *
    mul, down. Returns the fp32 output of down."""
    r = rms_norm_ref(x, norm_w, eps)
    h = silu_mul_ref(_proj_fp16(r, gate), _proj_fp16(r, up))
    return w4a16_linear_ref(h, *down)


def qkv_ref(x, norm_w, eps: float, q, k, v):
    """The q / k / v stage attention_forward_qkv_stage (fuse_v2/q_attn.cu:23-54):
    (RMSNorm output, fp32 q, k, v)."""
    r = rms_norm_ref(x, norm_w, eps)
    return r, w4a16_linear_ref(r, *q), w4a16_linear_ref(r, *k), w4a16_linear_ref(r, *v)
