"""Drop-in for the reference's Marlin GPTQ runtime (After-Revision-DROFELL/cuda_extends/
marlin.py): ``MarlinTuningParams``, ``MarlinDenseCache``, ``make_marlin_workspace``,
``MarlinQ4Matrix`` and the two autograd functions, with their names, arguments and
errors.

Marlin in the reference is the symmetric-only GPTQ backend: it refuses any zero point
other than 8 (every stored nibble 7, ``qzeros == 0x77777777``), repacks ``qweight`` into
its own tiled layout and multiplies with an SM80 ``mma.sync`` kernel below a token
threshold, or reconstructs the dense weight and calls cuBLAS above it.

Here a Marlin matrix is a handle of the same B200 kernels as ``Q4MatrixV2``, on the
unchanged GPTQ layout (the checkpoint's tensors are used as they are: no repack and
no re-export). The handle sees that every zero nibble is 7 and runs the symmetric
fast path: no kernel loads the zero points. Forward and backward never reconstruct a
dense weight and never call a dense library GEMM, for any number of tokens, so the
reconstruct thresholds of ``MarlinTuningParams`` are kept for callers that read them
but do not change the kernels.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
from torch.autograd import Function

from . import _capi

SYMMETRIC_ZERO_WORD = 0x77777777  # eight zero nibbles of 7: z = 8


@dataclass(frozen=True)
class MarlinTuningParams:
    """Token thresholds of the reference's dispatch (marlin.py:18-53; defaults measured
    there on an RTX 3090 for Llama-2-70B). ``use_reconstructed_forward`` answers as the
    reference does; the B200 path runs the packed-weight kernels at every size."""
    reconstruct_threshold: Optional[int] = 768
    grad_reconstruct_threshold: Optional[int] = 128
    reuse_reconstruct_cache_when_grad: Optional[bool] = None

    def __post_init__(self) -> None:
        for name in ("reconstruct_threshold", "grad_reconstruct_threshold"):
            value = getattr(self, name)
            if value is not None and value <= 0:
                raise ValueError(f"{name} must be positive or None")

    def use_reconstructed_forward(self, flattened_tokens: int, *, cache_weight: bool) -> bool:
        limit = self.grad_reconstruct_threshold if cache_weight else self.reconstruct_threshold
        return limit is not None and flattened_tokens >= limit

    def reuse_reconstruct_cache(self, default: bool) -> bool:
        if self.reuse_reconstruct_cache_when_grad is None:
            return default
        return self.reuse_reconstruct_cache_when_grad


class MarlinDenseCache:
    """The shared fp16 reconstruction buffer (interface of marlin.py:56-88): sized by the
    matrices that register, created once, then handed out as views. Nothing in this
    library's forward or backward uses it; ``MarlinQ4Matrix.reconstruct_weight`` fills
    views of it on request."""

    def __init__(self, device: torch.device) -> None:
        self.device = device
        self.temp_weight_elements = 0
        self._buf: Optional[torch.Tensor] = None

    def update(self, in_features: int, out_features: int) -> None:
        if self._buf is not None:
            raise RuntimeError("cannot resize initialized Marlin dense cache")
        self.temp_weight_elements = max(self.temp_weight_elements, in_features * out_features)

    def init_cache(self) -> None:
        if self._buf is not None:
            raise RuntimeError("Marlin dense cache initialized twice")
        self._buf = torch.empty(self.temp_weight_elements, dtype=torch.float16, device=self.device)

    def weight(self, in_features: int, out_features: int) -> torch.Tensor:
        if self._buf is None:
            raise RuntimeError("Marlin dense cache is not initialized")
        n = in_features * out_features
        if n > self._buf.numel():
            raise RuntimeError("Marlin dense cache is too small")
        return self._buf[:n].view(in_features, out_features)


def make_marlin_workspace(device: torch.device) -> torch.Tensor:
    """The per-matrix int32 workspace the reference's Marlin GEMM takes (marlin.py:90-96).
    The B200 kernels keep their own state, so it is only allocated (zeroed) to keep the
    module's buffers the same."""
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("Marlin workspace must be initialized on CUDA")
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return torch.zeros(sms * 4, dtype=torch.int32, device=device)


class MarlinQ4Matrix:
    """A symmetric GPTQ weight on the B200 kernels (interface of marlin.py:190-363).

    ``qweight`` / ``qzeros`` / ``scales`` stay the checkpoint's GPTQ tensors;
    ``g_idx_sort_indices`` is the act-order row sort (empty without act-order)."""

    def __init__(self, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, in_features: int,
                 out_features: int, g_idx: torch.Tensor, use_act_order: bool, workspace: torch.Tensor,
                 tuning_params: MarlinTuningParams, cache: MarlinDenseCache) -> None:
        if qweight.device.type != "cuda":
            raise ValueError("Marlin weights must be initialized on CUDA")
        if not bool((qzeros == SYMMETRIC_ZERO_WORD).all().item()):
            raise ValueError("Marlin requires symmetric GPTQ zero points")
        if workspace.device != qweight.device or workspace.dtype != torch.int32:
            raise ValueError("Marlin workspace has the wrong device or dtype")
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = in_features // scales.shape[0]
        self.use_act_order = use_act_order and self.group_size < in_features
        self.tuning_params = tuning_params
        self.cache = cache
        self.qweight = qweight.contiguous()
        self.qzeros = qzeros.contiguous()
        self.scales = scales.contiguous()
        self.g_idx = g_idx.to(device=qweight.device, dtype=torch.int32)
        if self.use_act_order:
            self.g_idx_sort_indices = torch.argsort(self.g_idx, stable=True).to(torch.int32)
        else:
            self.g_idx_sort_indices = torch.empty(0, dtype=torch.int32, device=qweight.device)
        self.workspace = workspace
        self._h = _capi.Handle(self.qweight, self.qzeros, self.scales,
                               self.g_idx.cpu() if self.use_act_order else None, qweight.device.index)
        assert self._h.symmetric, "the handle should have found the symmetric zero points"
        cache.update(in_features, out_features)

    def set_tuning_params(self, tuning_params: MarlinTuningParams) -> None:
        self.tuning_params = tuning_params

    def use_reconstructed_forward(self, flattened_tokens: int, *, cache_weight: bool) -> bool:
        return self.tuning_params.use_reconstructed_forward(flattened_tokens, cache_weight=cache_weight)

    def reconstruct_weight(self, output: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Dense fp16 W [K, N] = (q - 8) * s, bit-exact (the dequant kernel)."""
        if output is None:
            output = torch.empty((self.in_features, self.out_features), dtype=torch.float16, device=self.qweight.device)
        return self._h.dequant(output)

    def _packed(self, x: torch.Tensor, transposed: bool) -> torch.Tensor:
        k_in, k_out = (self.out_features, self.in_features) if transposed else (self.in_features, self.out_features)
        x2 = x.reshape(-1, k_in)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        out = torch.empty((x2.shape[0], k_out), dtype=x.dtype, device=x.device)
        if transposed:
            self._h.gemm_t(x2, out)
        else:
            self._h.gemm(x2, out)
        return out.view(*x.shape[:-1], k_out)

    def direct_matmul(self, x: torch.Tensor) -> torch.Tensor:
        """x [..., K] @ W on the packed weight (the reference's marlin_gemm)."""
        return self._packed(x, transposed=False)

    def dense_matmul(self, x: torch.Tensor, weight: torch.Tensor, *, transpose_weight: bool = False) -> torch.Tensor:
        """x @ weight (or weight^T) for a caller's dense fp16 weight (marlin.py:173-188)."""
        w = weight.t() if transpose_weight else weight
        x2 = x.reshape(-1, x.shape[-1])
        return torch.matmul(x2, w).view(*x.shape[:-1], w.shape[1])

    def forward_matmul(self, x: torch.Tensor, *, cache_weight: bool) -> tuple[torch.Tensor, Optional[torch.Tensor]]:
        """(x @ W, None): the packed-weight kernels at every size, so no dense weight is
        produced or kept for the backward."""
        return self.direct_matmul(x), None

    def transpose_matmul(self, x: torch.Tensor, weight: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x [..., N] @ W^T on the tcgen05 transposed GEMM. A cached dense ``weight`` is
        this matrix's reconstruction and gives the same product; it is not needed."""
        return self._packed(x, transposed=True)


class MarlinQ4LinearFunction(Function):
    """Autograd of a frozen Marlin matrix: only the input has a gradient (marlin.py:366-396)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, q4_matrix: MarlinQ4Matrix, cache_weight: bool) -> torch.Tensor:
        out, _ = q4_matrix.forward_matmul(x, cache_weight=cache_weight)
        ctx.q4_matrix = q4_matrix
        ctx.x_dtype = x.dtype
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        m: MarlinQ4Matrix = ctx.q4_matrix
        grad = m.transpose_matmul(grad_output.to(m.scales.dtype).contiguous())
        return grad.to(ctx.x_dtype), None, None


class MarlinQ4ForwardOnlyLinearFunction(Function):
    """Inference forward (marlin.py:401-413); it has no backward."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, q4_matrix: MarlinQ4Matrix) -> torch.Tensor:
        out, _ = q4_matrix.forward_matmul(x, cache_weight=False)
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        raise RuntimeError("MarlinQ4ForwardOnlyLinearFunction has no backward")
