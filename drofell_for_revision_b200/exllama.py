"""Drop-in for the reference's ExLlama-v2 W4A16 runtime module.

The reference module (After-Revision-DROFELL/cuda_extends/exllama.py) is the Python
face of its ``prebuilt_exllama_extend`` extension. The quantized-linear operator uses
these names from it, kept here with the same arguments, meaning and errors:
``TuningParams`` (:22-46), ``make_q4`` and the ``q4_*_v2`` entry points (:49-118,
entry.cpp:18-251), ``CacheV2`` (:358-378), ``Q4MatrixV2`` (:381-546) and the two
autograd functions (:649-740). ``RuntimeError`` is raised where the extension's
TORCH_CHECKs fail, ``AssertionError`` where the Python module asserts.

How this one works: every product is computed by the packed-weight kernels of the C
ABI (``_capi.Handle``): the decode GEMVs and the tcgen05 GEMM forward, the tcgen05
transposed GEMM backward. Nothing is reconstructed into a dense scratch weight and
no dense library GEMM is called, for any M, dtype or act-order table. A dense copy
of the weight exists only when a caller asks for one (the ``q4_to_*`` getters,
``reconstruct_weight``, or a ``temp_weight`` buffer it hands in to be filled).
The caller's packed tensors are never modified (the reference shuffles and row-sorts
``qweight`` in place, q4_matrix.cu:67-75,179).
"""
from __future__ import annotations

import weakref
from dataclasses import dataclass
from typing import Any, NewType, Optional, Tuple

import torch
from torch.autograd import Function

from . import _capi

Q4Ptr = NewType("Q4Ptr", int)


@dataclass
class TuningParams:
    """The reference's launch knobs (field names and defaults of exllama.py:22-46).

    Callers build and pass one; the B200 kernels plan their own launch shapes from the
    weight's shape and the SM count, so none of these values changes a launch here.
    ``GEMV_REPACK`` is this library's own knob: whether each matrix also keeps a copy of
    its weight in the order of the ``mma.sync`` decode GEMV (faster for 3 <= M <= 16, the
    same size as ``qweight``). It is read once, when the matrix is created."""
    RECONSTRUCT_THREADS_X: int = 128
    RECONSTRUCT_THREADS_Y: int = 1
    COLUMN_SHUFFLE_BLOCK_X: int = 256
    COLUMN_SHUFFLE_BLOCK_Y: int = 16
    MATMUL_THREADS_X: int = 32
    MATMUL_THREADS_Y: int = 1
    MATMUL_BLOCK_SIZE_Z: Optional[int] = None
    MATMUL_GROUP_STEP: int = 32
    MATMAL_RECONSTRUCT_THRESHOLD: int = 8
    MATMAL_RECONSTRUCT_THRESHOLD_V2: int = 50
    NO_HALF2: bool = False
    NO_FUSE_REMAP: bool = True
    BLOCK_KN_SIZE: int = 128
    BLOCK_M_SIZE_MAX: int = 8
    GEMV_REPACK: bool = True


# The reference hands raw Q4Matrix* integers between calls (entry.cpp:62); this maps the
# integer back to its Handle without keeping the Handle alive.
_HANDLES: "weakref.WeakValueDictionary[int, _capi.Handle]" = weakref.WeakValueDictionary()


def _handle(q4: int) -> _capi.Handle:
    h = _HANDLES.get(int(q4))
    if h is None:
        raise RuntimeError(f"unknown or released q4 handle {q4:#x}")
    return h


def make_q4(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, g_idx: Optional[torch.Tensor],
            cuda_x_map: Optional[torch.Tensor], device: int, use_act: bool, v2_mode: bool = True,
            repack: bool = True) -> "_capi.Handle":
    """Create the packed-weight handle (entry.cpp:18-62). Returns the owning Handle;
    ``int(handle.as_int)`` is the Q4Ptr other entry points accept.

    With ``use_act`` the stable group sort of the rows (the reference's x_map,
    q4_matrix.cu:125-176) is written into ``cuda_x_map`` as the reference does.
    ``repack=False`` skips the mma.sync-ordered weight copy (TuningParams.GEMV_REPACK)."""
    if qweight.dtype != torch.int32:
        raise RuntimeError("qweight must be torch.int32")
    if qzeros.dtype != torch.int32:
        raise RuntimeError("qzeros must be torch.int32")
    if scales.dtype != torch.float16:
        raise RuntimeError("scales must be torch.float16")
    height = qweight.shape[0] * 8
    if use_act:
        if g_idx is None or g_idx.dtype != torch.int32:
            raise RuntimeError("g_idx must be torch.int32")
        if cuda_x_map is not None and cuda_x_map.device.type != "meta":
            if cuda_x_map.dtype != torch.int32:
                raise RuntimeError("cuda_x_map must be torch.int32")
            if cuda_x_map.shape[0] != g_idx.shape[0] or height != cuda_x_map.shape[0]:
                raise RuntimeError("cuda_x_map/g_idx and w have incompatible shapes")
    if qweight.shape[1] != qzeros.shape[1] * 8:
        raise RuntimeError("qweight and qzeros have incompatible shapes")
    if scales.shape[1] != qweight.shape[1]:
        raise RuntimeError("scales and qweight have incompatible shapes")
    if qzeros.shape[0] != scales.shape[0]:
        raise RuntimeError("qzeros and scales have incompatible shapes")
    h = _capi.Handle(qweight, qzeros, scales, g_idx if use_act else None, device, repack=repack)
    if use_act and cuda_x_map is not None and cuda_x_map.device.type != "meta":
        perm = torch.argsort(g_idx.detach().to("cpu", torch.int64), stable=True).to(torch.int32)
        cuda_x_map.copy_(perm.to(cuda_x_map.device))
    _HANDLES[h.as_int] = h
    return h


def make_q4_py(qweight, qzeros, scales, g_idx, cuda_x_map, device_idx, use_act, v2_mode):
    return make_q4(qweight, qzeros, scales, g_idx, cuda_x_map, device_idx, use_act, v2_mode)


def _dense_into(q4: int, out: torch.Tensor, dtype: torch.dtype) -> None:
    if out.dtype != dtype:
        raise RuntimeError(f"out_weights must be {dtype}")
    _handle(q4).dequant(out)


def q4_to_half_matrix_v2(q4: int, out_matrix: torch.Tensor, block_kn_size: int = 128) -> None:
    """Dense fp16 W in original row order (entry.cpp:80-93)."""
    _dense_into(q4, out_matrix, torch.float16)


def q4_to_bfloat16_matrix_v2(q4: int, out_matrix: torch.Tensor, block_kn_size: int = 128) -> None:
    """Dense bf16 W = bf16(fp16 W) in original row order (entry.cpp:110-122)."""
    _dense_into(q4, out_matrix, torch.bfloat16)


def q4_to_half_matrix_v2_py(q4, out_matrix, BLOCK_KN_SIZE=128):
    return q4_to_half_matrix_v2(q4, out_matrix, BLOCK_KN_SIZE)


def q4_to_bfloat16_matrix_v2_py(q4, out_matrix, BLOCK_KN_SIZE=128):
    return q4_to_bfloat16_matrix_v2(q4, out_matrix, BLOCK_KN_SIZE)


def _check_x_out(x: torch.Tensor, out: torch.Tensor, in_features: int) -> None:
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("x must be float16 or bfloat16")
    if out.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("out must be float16 or bfloat16")
    if x.shape[0] != out.shape[0]:
        raise RuntimeError("x and out have incompatible shapes")
    if x.shape[-1] != in_features:
        raise RuntimeError("x and w have incompatible shapes")


def _fill_dense(h: _capi.Handle, temp_weight: Optional[torch.Tensor], dtype: torch.dtype) -> None:
    """The reference's reconstruct step leaves the dense weight in ``temp_weight``;
    callers that keep that buffer get it filled the same way."""
    if temp_weight is not None and temp_weight.numel() >= h.K * h.N and temp_weight.dtype == dtype:
        h.dequant(temp_weight.reshape(-1)[: h.K * h.N].view(h.K, h.N))


def q4_matmul_cuda_v2(x: torch.Tensor, q4: int, out: torch.Tensor, block_kn_size: int = 128,
                      block_m_size_max: int = 8, no_zero: bool = False) -> None:
    """out = x @ W (entry.cpp:221-251): the decode GEMV for M <= 16, the tcgen05 GEMM above."""
    h = _handle(q4)
    _check_x_out(x, out, h.K)
    if block_kn_size != 128:
        raise RuntimeError("currently support kn size = 128 only")
    h.gemm(x, out, _capi.PATH_AUTO)


def q4_matmul_blas_v2(x: torch.Tensor, q4: int, out: torch.Tensor, temp_weight: Optional[torch.Tensor],
                      no_zero: bool = False, block_kn_size: int = 128, skip_reconstruct: bool = False,
                      bfloat16: bool = False) -> None:
    """The reference's "reconstruct + cuBLAS" entry (q4_matmul.cu:459-510), computed by
    the tcgen05 GEMM on the packed weight. Without ``skip_reconstruct`` a full-size
    ``temp_weight`` is also filled with the dense weight, as the reference leaves it.
    With ``skip_reconstruct`` the reference multiplies by ``temp_weight``, which every
    one of its callers filled from this same matrix; the packed weight gives the same
    product, so it is used instead."""
    h = _handle(q4)
    _check_x_out(x, out, h.K)
    if (x.dtype == torch.bfloat16) != bfloat16:
        raise RuntimeError("x must be bfloat16" if bfloat16 else "x must be float16")
    if skip_reconstruct:
        assert temp_weight is not None
    else:
        _fill_dense(h, temp_weight, x.dtype)
    h.gemm(x, out, _capi.PATH_TC)


def q4_transpose_matmul_blas_v2(x: torch.Tensor, q4: int, out: torch.Tensor, temp_weight: Optional[torch.Tensor],
                                no_zero: bool = False, block_kn_size: int = 128, skip_reconstruct: bool = False,
                                bfloat16: bool = False) -> None:
    """out[M, K] = x[M, N] @ W^T for the PEFT backward (q4_transpose_matmul.cu:115-167),
    computed by the tcgen05 transposed GEMM on the packed weight (w4a16_gemm_t). The
    ``temp_weight`` / ``skip_reconstruct`` arguments behave as in q4_matmul_blas_v2."""
    h = _handle(q4)
    if x.shape[-1] != h.N:
        raise RuntimeError("x and w have incompatible shapes")
    if (x.dtype == torch.bfloat16) != bfloat16:
        raise RuntimeError("x must be bfloat16" if bfloat16 else "x must be float16")
    if skip_reconstruct:
        assert temp_weight is not None
    else:
        _fill_dense(h, temp_weight, x.dtype)
    h.gemm_t(x.reshape(-1, h.N), out.view(-1, h.K))


def q4_matmul_cuda_v2_py(x, q4, out, BLOCK_KN_SIZE=128, BLOCK_M_SIZE_MAX=8, no_zero=False):
    return q4_matmul_cuda_v2(x, q4, out, BLOCK_KN_SIZE, BLOCK_M_SIZE_MAX, no_zero)


def q4_matmul_blas_v2_py(x, q4, out, temp_weight, no_zero, BLOCK_KN_SIZE, skip_reconstruct, bfloat16):
    return q4_matmul_blas_v2(x, q4, out, temp_weight, no_zero, BLOCK_KN_SIZE, skip_reconstruct, bfloat16)


def q4_transpose_matmul_blas_v2_py(x, q4, out, temp_weight, no_zero, BLOCK_KN_SIZE, skip_reconstruct, bfloat16):
    return q4_transpose_matmul_blas_v2(x, q4, out, temp_weight, no_zero, BLOCK_KN_SIZE, skip_reconstruct, bfloat16)


def mlp_forward_v2(layernorm: torch.Tensor, norm_epsilon: float, gate_q4: int, up_q4: int, down_q4: int,
                   temp_rms_output: torch.Tensor, temp_gate_output: torch.Tensor, temp_up_output: torch.Tensor,
                   temp_weight: Optional[torch.Tensor], x: torch.Tensor, output: torch.Tensor,
                   block_kn_size: int = 128, block_m_size_max: int = 8, switch_threshold: int = 50) -> None:
    """The decoder MLP block (entry.cpp:431-481 -> fuse_v2/q_mlp.cu:96-133):
    output = down(silu(gate(r)) * up(r)) with r = RMSNorm(x; layernorm, norm_epsilon) left
    in ``temp_rms_output``. At decode sizes (one or two rows) it is two kernel launches
    with the RMSNorm and the silu * mul applied while each GEMV stages its input; the
    reference runs five. ``temp_gate_output`` / ``temp_up_output`` are scratch of the block
    (their contents afterwards are unspecified); ``temp_weight`` and the tuning values are
    accepted and unused."""
    if layernorm.dtype != torch.float16:
        raise RuntimeError("layernorm weight must be float16 or bfloat16")
    _capi.mlp_forward(_handle(gate_q4), _handle(up_q4), _handle(down_q4), layernorm, norm_epsilon, x, output,
                      temp_rms_output, temp_gate_output, temp_up_output)


def attention_forward_qkv_stage_v2(layernorm: torch.Tensor, norm_epsilon: float, q_proj: int, k_proj: int,
                                   v_proj: int, temp_rms_output: torch.Tensor, temp_q_output: torch.Tensor,
                                   temp_k_output: torch.Tensor, temp_v_output: torch.Tensor,
                                   temp_weight: Optional[torch.Tensor], x: torch.Tensor, block_kn_size: int,
                                   block_m_size_max: int, switch_threshold: int, q_len: int, batch_size: int) -> None:
    """The attention input stage (entry.cpp:483-532 -> fuse_v2/q_attn.cu:23-54): r =
    RMSNorm(x) into ``temp_rms_output`` and the q, k, v projections of r into the three
    output buffers, for ``q_len * batch_size`` rows. At decode sizes it is one launch over
    the three weights with the RMSNorm applied while X is staged (the reference: four)."""
    if layernorm.dtype != torch.float16:
        raise RuntimeError("layernorm weight must be float16 or bfloat16")
    rows = q_len * batch_size
    hq = _handle(q_proj)
    _capi.qkv_forward(hq, _handle(k_proj), _handle(v_proj), layernorm, norm_epsilon, x.reshape(-1, hq.K)[:rows],
                      temp_rms_output, temp_q_output, temp_k_output, temp_v_output)


def mlp_forward_v2_py(layernorm, norm_epsilon, gate_q4, up_q4, down_q4, temp_rms_output, temp_gate_output,
                      temp_up_output, temp_weight, x, output, BLOCK_KN_SIZE, BLOCK_M_SIZE_MAX,
                      MATMAL_RECONSTRUCT_THRESHOLD_V2):
    return mlp_forward_v2(layernorm, norm_epsilon, gate_q4, up_q4, down_q4, temp_rms_output, temp_gate_output,
                          temp_up_output, temp_weight, x, output, BLOCK_KN_SIZE, BLOCK_M_SIZE_MAX,
                          MATMAL_RECONSTRUCT_THRESHOLD_V2)


def attention_forward_qkv_stage_v2_py(layernorm, norm_epsilon, q_proj, k_proj, v_proj, temp_rms_output,
                                      temp_q_output, temp_k_output, temp_v_output, temp_weight, x, BLOCK_KN_SIZE,
                                      BLOCK_M_SIZE_MAX, MATMAL_RECONSTRUCT_THRESHOLD_V2, q_len, bsz):
    return attention_forward_qkv_stage_v2(layernorm, norm_epsilon, q_proj, k_proj, v_proj, temp_rms_output,
                                          temp_q_output, temp_k_output, temp_v_output, temp_weight, x,
                                          BLOCK_KN_SIZE, BLOCK_M_SIZE_MAX, MATMAL_RECONSTRUCT_THRESHOLD_V2,
                                          q_len, bsz)


class CacheV2:
    """The shared fp16 scratch ``post_init`` hands every matrix (API of exllama.py:358-378).

    The reference reconstructs each weight into this buffer before a cuBLAS GEMM. The
    kernels here read the packed weight directly, so nothing in this library writes to
    it; it is kept so that code which sizes, creates and reads it works unchanged.
    Matrices register the elements they would need; ``init_cache`` allocates that many,
    and a later, larger registration invalidates the buffer until the next
    ``init_cache``."""

    def __init__(self, device: torch.device) -> None:
        self.device: torch.device = device
        self._need = 0
        self._buf: Optional[torch.Tensor] = None

    @property
    def temp_weight_size(self) -> int:
        return self._need

    @property
    def cache_created(self) -> bool:
        return self._buf is not None and self._buf.shape[1] >= self._need

    def update_temp_weight_size(self, temp_weight_size: int) -> None:
        self._need = max(self._need, int(temp_weight_size))

    def init_cache(self) -> None:
        self._buf = torch.empty((1, self._need), dtype=torch.float16, device=self.device)

    @property
    def temp_weight(self) -> torch.Tensor:
        assert self.cache_created, "CacheV2.init_cache() has not been called since the last size update"
        return self._buf


class Q4MatrixV2:
    """A packed GPTQ weight bound to the B200 kernels (interface of exllama.py:381-546).

    ``height`` = in_features K, ``width`` = out_features N. ``cuda_q4`` is the integer
    handle the reference's fused entry points take. Dense copies of the weight are kept
    only on request (``reconstruct_weight``) and never used for products."""

    def __init__(self, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, height: int, width: int,
                 g_idx: Optional[torch.Tensor], use_act: bool, tuning_params: TuningParams, cache: CacheV2) -> None:
        if use_act:
            assert g_idx is not None
        self.use_act = use_act
        self.height, self.width = height, width
        self.device = qweight.device
        self.tuning_params = tuning_params
        self.cache = cache
        self.cuda_x_map: Optional[torch.Tensor] = (
            torch.zeros(g_idx.shape, dtype=torch.int32, device=self.device) if use_act else None)
        self._h = make_q4(qweight, qzeros, scales, g_idx if use_act else None, self.cuda_x_map, self.device.index,
                          use_act, True, repack=getattr(tuning_params, "GEMV_REPACK", True))
        assert (self._h.K, self._h.N) == (height, width), "height/width disagree with qweight"
        self.cuda_q4: Q4Ptr = Q4Ptr(self._h.as_int)
        cache.update_temp_weight_size(height * width)
        self._kept: dict = {torch.float16: None, torch.bfloat16: None}

    # dense copies kept on request (attribute names of the reference)
    @property
    def reconstructed_weight_float16(self) -> Optional[torch.Tensor]:
        return self._kept[torch.float16]

    @property
    def reconstructed_weight_bfloat16(self) -> Optional[torch.Tensor]:
        return self._kept[torch.bfloat16]

    def dense(self, dtype: torch.dtype, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """W [K, N] in original row order, fp16 or bf16 (bit-exact dequant kernel)."""
        if out is None:
            out = torch.empty((self.height, self.width), dtype=dtype, device=self.device)
        _dense_into(self.cuda_q4, out, dtype)
        return out

    def get_float16_weights_matrix_v2(self, out_matrix: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.dense(torch.float16, out_matrix)

    def get_bfloat16_weights_matrix_v2(self, out_matrix: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.dense(torch.bfloat16, out_matrix)

    def reconstruct_weight(self, dtype: torch.dtype) -> None:
        assert dtype in self._kept
        self._kept[dtype] = self.dense(dtype)

    def release_weight(self, dtype: Optional[torch.dtype] = None) -> None:
        for dt in (list(self._kept) if dtype is None else [dtype]):
            if dt in self._kept:
                self._kept[dt] = None

    def set_tuning_params(self, tuning_params: TuningParams) -> None:
        self.tuning_params = tuning_params

    def get_weight_matrix_shape(self) -> Tuple[int, int]:
        return (self.height, self.width)

    def get_x_features(self) -> int:
        return max(self.height, self.width)

    def _apply(self, x: torch.Tensor, output: Optional[torch.Tensor], features_out: int, transposed: bool):
        assert x.dtype in (torch.float16, torch.bfloat16), f"{x.dtype}"
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        if output is None:
            output = torch.empty((x2.shape[0], features_out), dtype=x.dtype, device=x.device)
        out2 = output.view(-1, features_out)
        if transposed:
            self._h.gemm_t(x2, out2)
        else:
            self._h.gemm(x2, out2, _capi.PATH_AUTO)
        return output.view(*lead, features_out)

    def matmul(self, x: torch.Tensor, output: Optional[torch.Tensor], temp_weight: Optional[torch.Tensor],
               must_blas: bool = False) -> torch.Tensor:
        """x [..., K] @ W -> [..., N] on the packed-weight kernels. ``temp_weight``, when
        given, is filled with the dense weight (the reference's reconstruct leaves it so)."""
        _fill_dense(self._h, temp_weight, x.dtype)
        return self._apply(x, output, self.width, transposed=False)

    def transpose_matmul(self, x: torch.Tensor, output: Optional[torch.Tensor], temp_weight: Optional[torch.Tensor],
                         skip_reconstruct: bool = False) -> torch.Tensor:
        """x [..., N] @ W^T -> [..., K] (the input gradient) on the tcgen05 transposed GEMM."""
        return self._apply(x, output, self.height, transposed=True)


def _linear_forward(weight_q4: Q4MatrixV2, x: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
    y = weight_q4.matmul(x, None, None)
    if bias is not None:
        y += bias
    return y


class ExllamaQ4LinearFunction(Function):
    """Y = X W (+ bias) with the input gradient dX = dY W^T (exllama.py:649-696).

    The packed weight is frozen, so only the input has a gradient. ``cache_weight`` is
    accepted for the reference's signature: the reference keeps a dense copy of W for
    the backward, but the transposed kernel here reads the packed weight, so nothing is
    kept between forward and backward."""

    @staticmethod
    def forward(ctx: Any, input: torch.Tensor, weight_q4: Q4MatrixV2, bias: Optional[torch.Tensor],
                cache_weight: bool) -> torch.Tensor:  # type: ignore[override]
        ctx.weight_q4 = weight_q4
        return _linear_forward(weight_q4, input, bias)

    @staticmethod
    def backward(ctx: Any, grad_output: torch.Tensor) -> Tuple[Optional[torch.Tensor], None, None, None]:  # type: ignore[override]
        if not ctx.needs_input_grad[0]:
            return None, None, None, None
        return ctx.weight_q4.transpose_matmul(grad_output, None, None), None, None, None


class ExllamaQ4ForwardOnlyLinearFunction(Function):
    """Inference forward (exllama.py:730-740); its backward yields no gradients."""

    @staticmethod
    def forward(ctx: Any, input: torch.Tensor, weight_q4: Q4MatrixV2,
                bias: Optional[torch.Tensor]) -> torch.Tensor:  # type: ignore[override]
        return _linear_forward(weight_q4, input, bias)

    @staticmethod
    def backward(ctx: Any, grad_output: torch.Tensor) -> Tuple[None, None, None]:  # type: ignore[override]
        return None, None, None
