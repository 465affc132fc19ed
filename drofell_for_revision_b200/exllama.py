"""Drop-in for the reference's ExLlama-v2 W4A16 runtime module.

Mirrors the public surface of After-Revision-DROFELL/cuda_extends/exllama.py that
the quantized-linear operator uses: ``TuningParams`` (:22-46), ``make_q4`` and the
v2 kernels' Python entry points (:49-118), ``CacheV2`` (:358-378), ``Q4MatrixV2``
(:381-546) and the autograd functions (:649-740). Same names, argument meaning
and error behaviour (``RuntimeError`` for what the reference's TORCH_CHECKs
reject, ``AssertionError`` for its Python asserts).

Differences, all on purpose:
  * the packed tensors are never modified (the reference shuffles and row-sorts
    ``qweight`` in place, q4_matrix.cu:67-75,179);
  * ``q4_matmul_cuda_v2`` / ``q4_matmul_blas_v2`` run the B200 kernels of the C ABI
    (CUDA-core GEMV for small fp16 M, tcgen05 tensor-core GEMM otherwise) for any M
    and both fp16 and bf16; nothing is reconstructed into a dense scratch weight;
  * ``CacheV2`` is accepted and kept, but its scratch buffer is no longer needed by
    the forward path.
"""
from __future__ import annotations

import weakref
from dataclasses import dataclass
from typing import Any, NewType, Optional, Tuple, Union

import torch
from torch.autograd import Function

from . import _capi

Q4Ptr = NewType("Q4Ptr", int)


@dataclass
class TuningParams:
    """Reference tuning knobs (exllama.py:22-46). Accepted for compatibility; the
    B200 kernels choose their own launch shapes. ``MATMAL_RECONSTRUCT_THRESHOLD_V2``
    is unused: there is no reconstruct path to switch to."""
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


# handle registry: the reference passes raw Q4Matrix* integers around (entry.cpp:62)
_HANDLES: "weakref.WeakValueDictionary[int, _capi.Handle]" = weakref.WeakValueDictionary()


def _handle(q4: int) -> _capi.Handle:
    h = _HANDLES.get(int(q4))
    if h is None:
        raise RuntimeError(f"unknown or released q4 handle {q4:#x}")
    return h


def make_q4(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, g_idx: Optional[torch.Tensor],
            cuda_x_map: Optional[torch.Tensor], device: int, use_act: bool, v2_mode: bool = True) -> "_capi.Handle":
    """Create the packed-weight handle (entry.cpp:18-62). Returns the owning Handle;
    ``int(handle.as_int)`` is the Q4Ptr other entry points accept.

    With ``use_act`` the stable group sort of the rows (the reference's x_map,
    q4_matrix.cu:125-176) is written into ``cuda_x_map`` as the reference does."""
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
    h = _capi.Handle(qweight, qzeros, scales, g_idx if use_act else None, device)
    if use_act and cuda_x_map is not None and cuda_x_map.device.type != "meta":
        perm = torch.argsort(g_idx.detach().to("cpu", torch.int64), stable=True).to(torch.int32)
        cuda_x_map.copy_(perm.to(cuda_x_map.device))
    _HANDLES[h.as_int] = h
    return h


def make_q4_py(qweight, qzeros, scales, g_idx, cuda_x_map, device_idx, use_act, v2_mode):
    return make_q4(qweight, qzeros, scales, g_idx, cuda_x_map, device_idx, use_act, v2_mode)


def q4_to_half_matrix_v2(q4: int, out_matrix: torch.Tensor, block_kn_size: int = 128) -> None:
    """Dense fp16 W in original row order (entry.cpp:80-93)."""
    if out_matrix.dtype != torch.float16:
        raise RuntimeError("out_weights must be torch.float16")
    _handle(q4).dequant(out_matrix)


def q4_to_bfloat16_matrix_v2(q4: int, out_matrix: torch.Tensor, block_kn_size: int = 128) -> None:
    """Dense bf16 W = bf16(fp16 W) in original row order (entry.cpp:110-122)."""
    if out_matrix.dtype != torch.bfloat16:
        raise RuntimeError("out_weights must be torch.bfloat16")
    _handle(q4).dequant(out_matrix)


def q4_to_half_matrix_v2_py(q4, out_matrix, BLOCK_KN_SIZE=128):
    return q4_to_half_matrix_v2(q4, out_matrix, BLOCK_KN_SIZE)


def q4_to_bfloat16_matrix_v2_py(q4, out_matrix, BLOCK_KN_SIZE=128):
    return q4_to_bfloat16_matrix_v2(q4, out_matrix, BLOCK_KN_SIZE)


def _check_x_out(x: torch.Tensor, out: torch.Tensor, h: _capi.Handle) -> None:
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("x must be float16 or bfloat16")
    if out.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("out must be float16 or bfloat16")
    if x.shape[0] != out.shape[0]:
        raise RuntimeError("x and out have incompatible shapes")
    if x.shape[-1] != h.K:
        raise RuntimeError("x and w have incompatible shapes")


def q4_matmul_cuda_v2(x: torch.Tensor, q4: int, out: torch.Tensor, block_kn_size: int = 128,
                      block_m_size_max: int = 8, no_zero: bool = False) -> None:
    """out = x @ W for the decode path (entry.cpp:221-251): the CUDA-core GEMV for small
    fp16 M, the tensor-core GEMM otherwise."""
    h = _handle(q4)
    _check_x_out(x, out, h)
    if block_kn_size != 128:
        raise RuntimeError("currently support kn size = 128 only")
    h.gemm(x, out, _capi.PATH_AUTO)


def q4_matmul_blas_v2(x: torch.Tensor, q4: int, out: torch.Tensor, temp_weight: Optional[torch.Tensor],
                      no_zero: bool = False, block_kn_size: int = 128, skip_reconstruct: bool = False,
                      bfloat16: bool = False) -> None:
    """The reference's "reconstruct + cuBLAS" entry (q4_matmul.cu:459-510).

    ``skip_reconstruct`` with a dense ``temp_weight`` keeps the reference behaviour
    (a plain dense GEMM on the caller's weight, through torch/cuBLAS). Otherwise the
    packed weight is multiplied directly by the tensor-core kernel, and if a
    ``temp_weight`` buffer of the full [K, N] shape is supplied it is also filled
    with the dequantized weight, as the reference's reconstruct step leaves it."""
    h = _handle(q4)
    _check_x_out(x, out, h)
    if (x.dtype == torch.bfloat16) != bfloat16:
        raise RuntimeError("x must be bfloat16" if bfloat16 else "x must be float16")
    if skip_reconstruct:
        assert temp_weight is not None
        torch.matmul(x, temp_weight.view(h.K, h.N).to(x.dtype), out=out)
        return
    if temp_weight is not None and temp_weight.numel() == h.K * h.N and temp_weight.dtype == x.dtype:
        h.dequant(temp_weight.view(h.K, h.N))
    h.gemm(x, out, _capi.PATH_TC if x.shape[0] > 0 else _capi.PATH_AUTO)


def q4_transpose_matmul_blas_v2(x: torch.Tensor, q4: int, out: torch.Tensor, temp_weight: Optional[torch.Tensor],
                                no_zero: bool = False, block_kn_size: int = 128, skip_reconstruct: bool = False,
                                bfloat16: bool = False) -> None:
    """out[M, K] = x[M, N] @ W^T for PEFT backward (q4_transpose_matmul.cu:115-167):
    dequantize (unless ``skip_reconstruct``) and multiply with a dense GEMM."""
    h = _handle(q4)
    if x.shape[-1] != h.N:
        raise RuntimeError("x and w have incompatible shapes")
    if skip_reconstruct:
        assert temp_weight is not None
        w = temp_weight.view(h.K, h.N)
    else:
        if temp_weight is not None and temp_weight.numel() >= h.K * h.N and temp_weight.dtype == x.dtype:
            w = temp_weight.reshape(-1)[: h.K * h.N].view(h.K, h.N)
        else:
            w = torch.empty((h.K, h.N), dtype=x.dtype, device=x.device)
        h.dequant(w)
    torch.matmul(x, w.t().to(x.dtype), out=out)


def q4_matmul_cuda_v2_py(x, q4, out, BLOCK_KN_SIZE=128, BLOCK_M_SIZE_MAX=8, no_zero=False):
    return q4_matmul_cuda_v2(x, q4, out, BLOCK_KN_SIZE, BLOCK_M_SIZE_MAX, no_zero)


def q4_matmul_blas_v2_py(x, q4, out, temp_weight, no_zero, BLOCK_KN_SIZE, skip_reconstruct, bfloat16):
    return q4_matmul_blas_v2(x, q4, out, temp_weight, no_zero, BLOCK_KN_SIZE, skip_reconstruct, bfloat16)


def q4_transpose_matmul_blas_v2_py(x, q4, out, temp_weight, no_zero, BLOCK_KN_SIZE, skip_reconstruct, bfloat16):
    return q4_transpose_matmul_blas_v2(x, q4, out, temp_weight, no_zero, BLOCK_KN_SIZE, skip_reconstruct, bfloat16)


class CacheV2(object):
    """Shared scratch of the reference (exllama.py:358-378), kept for API compatibility."""

    def __init__(self, device: torch.device) -> None:
        self.temp_weight_size: int = 0
        self._temp_weight: Optional[torch.Tensor] = None
        self.device: torch.device = device
        self.cache_created = False

    def update_temp_weight_size(self, temp_weight_size: int):
        if temp_weight_size > self.temp_weight_size:
            self.cache_created = False
            self.temp_weight_size = temp_weight_size

    @property
    def temp_weight(self) -> torch.Tensor:
        assert self.cache_created
        assert self._temp_weight is not None
        return self._temp_weight

    def init_cache(self):
        self._temp_weight = torch.empty(size=(1, self.temp_weight_size), dtype=torch.float16, requires_grad=False,
                                        device=self.device)
        self.cache_created = True


class Q4MatrixV2(object):
    """The packed-weight object of exllama.py:381-546, backed by the B200 C ABI."""

    def __init__(self, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, height: int, width: int,
                 g_idx: Optional[torch.Tensor], use_act: bool, tuning_params: TuningParams, cache: CacheV2) -> None:
        self.use_act = use_act
        self.cuda_x_map: Optional[torch.Tensor] = None
        if self.use_act:
            assert g_idx is not None
            self.cuda_x_map = torch.zeros(size=g_idx.size(), dtype=g_idx.dtype, device=qweight.device)
        self._h = make_q4(qweight, qzeros, scales, g_idx if use_act else None, self.cuda_x_map,
                          qweight.device.index, use_act, True)
        self.cuda_q4: Q4Ptr = Q4Ptr(self._h.as_int)
        self.height = height
        self.width = width
        self.device = qweight.device
        self.tuning_params = tuning_params
        self.cache = cache
        cache.update_temp_weight_size(qweight.numel() * 8)
        self.reconstructed_weight_float16: Optional[torch.Tensor] = None
        self.reconstructed_weight_bfloat16: Optional[torch.Tensor] = None
        assert self._h.K == height and self._h.N == width, "height/width disagree with qweight"

    def reconstruct_weight(self, dtype: torch.dtype):
        assert dtype in [torch.float16, torch.bfloat16]
        if dtype == torch.float16:
            self.reconstructed_weight_float16 = self.get_float16_weights_matrix_v2()
        else:
            self.reconstructed_weight_bfloat16 = self.get_bfloat16_weights_matrix_v2()

    def release_weight(self, dtype: Optional[torch.dtype] = None):
        if dtype is None:
            self.reconstructed_weight_float16 = None
            self.reconstructed_weight_bfloat16 = None
        elif dtype == torch.float16:
            self.reconstructed_weight_float16 = None
        elif dtype == torch.bfloat16:
            self.reconstructed_weight_bfloat16 = None

    def set_tuning_params(self, tuning_params: TuningParams):
        self.tuning_params = tuning_params

    def get_weight_matrix_shape(self):
        return (self.height, self.width)

    def get_x_features(self):
        return max(self.height, self.width)

    def get_float16_weights_matrix_v2(self, out_matrix: Optional[torch.Tensor] = None):
        if out_matrix is None:
            out_matrix = torch.empty(self.height, self.width, dtype=torch.half, device=self.device)
        q4_to_half_matrix_v2(self.cuda_q4, out_matrix, self.tuning_params.BLOCK_KN_SIZE)
        return out_matrix

    def get_bfloat16_weights_matrix_v2(self, out_matrix: Optional[torch.Tensor] = None):
        if out_matrix is None:
            out_matrix = torch.empty(self.height, self.width, dtype=torch.bfloat16, device=self.device)
        q4_to_bfloat16_matrix_v2(self.cuda_q4, out_matrix, self.tuning_params.BLOCK_KN_SIZE)
        return out_matrix

    def matmul(self, x: torch.Tensor, output: Optional[torch.Tensor], temp_weight: Optional[torch.Tensor],
               must_blas: bool = False):
        assert x.dtype == torch.float16 or x.dtype == torch.bfloat16, f"{x.dtype}"
        outshape = x.shape[:-1] + (self.width,)
        x = x.reshape(-1, x.shape[-1])
        if not x.is_contiguous():
            x = x.contiguous()
        x_height = x.shape[0]
        if output is None:
            output = torch.empty((x_height, self.width), dtype=x.dtype, device=x.device,
                                 requires_grad=x.requires_grad)
        if x.dtype == torch.float16 and self.reconstructed_weight_float16 is not None:
            q4_matmul_blas_v2(x, self.cuda_q4, output, self.reconstructed_weight_float16, False,
                              self.tuning_params.BLOCK_KN_SIZE, True, False)
            return output.view(outshape)
        elif x.dtype == torch.bfloat16 and self.reconstructed_weight_bfloat16 is not None:
            q4_matmul_blas_v2(x, self.cuda_q4, output, self.reconstructed_weight_bfloat16, False,
                              self.tuning_params.BLOCK_KN_SIZE, True, True)
            return output.view(outshape)
        if must_blas and temp_weight is not None:
            q4_matmul_blas_v2(x, self.cuda_q4, output, temp_weight, False, self.tuning_params.BLOCK_KN_SIZE, False,
                              x.dtype == torch.bfloat16)
        else:
            try:
                self._h.gemm(x, output, _capi.PATH_AUTO)
            except _capi.W4A16Error as e:
                if e.code != _capi.W4A16_ERR_UNSUPPORTED:
                    raise
                # act-order groups that do not fill whole 8-row words: dequant kernel + dense GEMM
                w = torch.empty((self.height, self.width), dtype=x.dtype, device=x.device)
                self._h.dequant(w)
                torch.matmul(x, w, out=output)
        return output.view(outshape)

    def transpose_matmul(self, x: torch.Tensor, output: Optional[torch.Tensor], temp_weight: Optional[torch.Tensor],
                         skip_reconstruct: bool = False):
        assert x.dtype == torch.float16 or x.dtype == torch.bfloat16
        outshape = x.shape[:-1] + (self.height,)
        x = x.reshape(-1, x.shape[-1])
        x_height = x.shape[0]
        if output is None:
            output = torch.empty((x_height, self.height), dtype=x.dtype, device=x.device,
                                 requires_grad=x.requires_grad)
        if x.dtype == torch.float16 and self.reconstructed_weight_float16 is not None:
            q4_transpose_matmul_blas_v2(x, self.cuda_q4, output, self.reconstructed_weight_float16, False,
                                        self.tuning_params.BLOCK_KN_SIZE, True, False)
            return output.view(outshape)
        elif x.dtype == torch.bfloat16 and self.reconstructed_weight_bfloat16 is not None:
            q4_transpose_matmul_blas_v2(x, self.cuda_q4, output, self.reconstructed_weight_bfloat16, False,
                                        self.tuning_params.BLOCK_KN_SIZE, True, True)
            return output.view(outshape)
        q4_transpose_matmul_blas_v2(x, self.cuda_q4, output, temp_weight, False, self.tuning_params.BLOCK_KN_SIZE,
                                    skip_reconstruct, x.dtype == torch.bfloat16)
        return output.view(outshape)


class ExllamaQ4LinearFunction(Function):
    """Forward + input-grad backward (exllama.py:649-696)."""

    @staticmethod
    def forward(ctx: Any, input: torch.Tensor, weight_q4: Q4MatrixV2, bias: Optional[torch.Tensor],
                cache_weight: bool) -> torch.Tensor:  # type: ignore[override]
        ctx.weight_q4 = weight_q4
        if cache_weight:
            if input.dtype == torch.float16 and (weight_q4.reconstructed_weight_float16 is not None):
                cache_weight = False
            elif input.dtype == torch.bfloat16 and (weight_q4.reconstructed_weight_bfloat16 is not None):
                cache_weight = False
        ctx.cache_weight = cache_weight
        if cache_weight:
            weight_restored = torch.empty(weight_q4.get_weight_matrix_shape(), requires_grad=False,
                                          device=weight_q4.device, dtype=input.dtype)
            output = weight_q4.matmul(input, output=None, temp_weight=weight_restored, must_blas=True)
            ctx.save_for_backward(weight_restored)
        else:
            output = weight_q4.matmul(input, output=None, temp_weight=None, must_blas=False)
        if bias is not None:
            output += bias.unsqueeze(0).expand_as(output)
        return output

    @staticmethod
    def backward(ctx: Any, grad_output: torch.Tensor) -> Tuple[Optional[torch.Tensor], None, None, None]:  # type: ignore[override]
        grad_input = None
        if ctx.needs_input_grad[0]:
            cached_weight = None
            if ctx.cache_weight:
                cached_weight, = ctx.saved_tensors
            weight_q4: Q4MatrixV2 = ctx.weight_q4
            grad_input = weight_q4.transpose_matmul(grad_output.contiguous(), output=None, temp_weight=cached_weight,
                                                    skip_reconstruct=cached_weight is not None)
        return grad_input, None, None, None


class ExllamaQ4ForwardOnlyLinearFunction(Function):
    """Inference forward (exllama.py:730-740)."""

    @staticmethod
    def forward(ctx: Any, input: torch.Tensor, weight_q4: Q4MatrixV2,
                bias: Optional[torch.Tensor]) -> torch.Tensor:  # type: ignore[override]
        output = weight_q4.matmul(input, None, None, False)
        if bias is not None:
            output += bias.unsqueeze(0).expand_as(output)
        return output

    @staticmethod
    def backward(ctx: Any, grad_output: torch.Tensor) -> Tuple[None, None, None]:  # type: ignore[override]
        return None, None, None
