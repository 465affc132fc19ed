"""Drop-in for the reference's Marlin quantized-linear operator
(After-Revision-DROFELL/operators/core/linear/real_marlin.py): ``MarlinQuantLinear`` and
``MarlinQuantLinearMaker`` with the same constructor arguments, registered buffers
(GPTQ ``qweight`` / ``qzeros`` / ``scales`` / ``g_idx`` as the checkpoint stores them, and
the non-persistent ``workspace``), errors and ``merge``.

Difference on purpose: ``post_init`` keeps the GPTQ tensors as they are (the reference
replaces them with Marlin's repacked ``qweight`` [K/16, 2N] and permuted ``scales``);
the B200 kernels read the GPTQ layout directly, with the symmetric fast path.
"""
from __future__ import annotations

import math
from typing import Optional, cast

import torch
from torch import nn

from . import flags
from .marlin import (MarlinDenseCache, MarlinQ4ForwardOnlyLinearFunction, MarlinQ4LinearFunction, MarlinQ4Matrix,
                     MarlinTuningParams, make_marlin_workspace)
from .real_quant import Linear, LinearMaker


class MarlinQuantLinear(Linear):
    """Symmetric GPTQ linear on the B200 kernels (interface of real_marlin.py:24-157)."""

    def __init__(self, group_size: int, in_features: int, out_features: int, bias: bool, use_act_order: bool) -> None:
        nn.Module.__init__(self)
        if bias:
            raise ValueError("the Marlin decode backend does not support bias")
        if in_features % 32 != 0 or out_features % 32 != 0:
            raise ValueError("Marlin GPTQ dimensions must be multiples of 32")
        self.infeatures = in_features
        self.outfeatures = out_features
        self.group_size = in_features if group_size == -1 else group_size
        if in_features % self.group_size != 0:
            raise ValueError("in_features must be divisible by group_size")
        self.use_act_order = use_act_order and self.group_size < in_features
        groups = math.ceil(in_features / self.group_size)
        self.register_buffer("qweight", torch.zeros((in_features // 8, out_features), dtype=torch.int32))
        self.register_buffer("qzeros", torch.zeros((groups, out_features // 8), dtype=torch.int32))
        self.register_buffer("scales", torch.zeros((groups, out_features), dtype=torch.float16))
        self.register_buffer("g_idx", (torch.arange(in_features) // self.group_size).to(torch.int32))
        # the reference allocates the workspace where the module is built; on a CPU module
        # it is made when the module reaches a GPU (post_init)
        self.register_buffer("workspace", None, persistent=False)
        self.bias = None
        self.q4_matrix: Optional[MarlinQ4Matrix] = None

    def post_init(self, tuning_params: MarlinTuningParams, cache: MarlinDenseCache) -> None:
        if self.q4_matrix is not None:
            raise RuntimeError("MarlinQuantLinear.post_init called twice")
        if self.workspace is None or self.workspace.device != self.qweight.device:
            self.workspace = make_marlin_workspace(self.qweight.device)
        m = MarlinQ4Matrix(self.qweight, self.qzeros, self.scales, self.infeatures, self.outfeatures, self.g_idx,
                           self.use_act_order, self.workspace, tuning_params, cache)
        self.register_buffer("g_idx_sort_indices", m.g_idx_sort_indices)
        self.q4_matrix = m

    def _matrix(self) -> MarlinQ4Matrix:
        if self.q4_matrix is None:
            raise RuntimeError("MarlinQuantLinear must be repacked before use")
        return self.q4_matrix

    @property
    def tuning_params(self) -> MarlinTuningParams:
        return self._matrix().tuning_params

    def reconstruct_weight(self, output: torch.Tensor) -> torch.Tensor:
        return self._matrix().reconstruct_weight(output)

    def dense_forward(self, x: torch.Tensor, dense_weight: torch.Tensor) -> torch.Tensor:
        return self._matrix().dense_matmul(x, dense_weight)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Y = X W in fp16 (X is cast to the scales' dtype and Y back, real_marlin.py:139-157)."""
        m = self._matrix()
        dtype_in = x.dtype
        xm = x.to(m.scales.dtype)
        if torch.is_grad_enabled() and xm.requires_grad:
            cache = m.tuning_params.reuse_reconstruct_cache(flags.REUSE_RECONSTRUCT_CACHE_WHEN_GRAD)
            y = MarlinQ4LinearFunction.apply(xm, m, cache)
        else:
            y = MarlinQ4ForwardOnlyLinearFunction.apply(xm, m)
        return cast(torch.Tensor, y).to(dtype_in)


class MarlinQuantLinearMaker(LinearMaker):
    """Builds, merges and finishes the model's Marlin layers (real_marlin.py:160-249)."""

    def __init__(self, quantization_group_size: int, use_act_order: bool) -> None:
        self.quantization_group_size = quantization_group_size
        self.use_act_order = use_act_order
        self.quant_linears: list[MarlinQuantLinear] = []
        self.post_inited = False

    def make_linear(self, in_features: int, out_features: int, bias: bool = False) -> MarlinQuantLinear:
        layer = MarlinQuantLinear(self.quantization_group_size, in_features, out_features, bias, self.use_act_order)
        self.quant_linears.append(layer)
        return layer

    def post_init(self, tuning_params: MarlinTuningParams, shared_cache: MarlinDenseCache) -> "MarlinQuantLinearMaker":
        if self.post_inited:
            raise RuntimeError("MarlinQuantLinearMaker.post_init called twice")
        if not self.quant_linears:
            raise RuntimeError("Marlin maker contains no quantized linears")
        self.post_inited = True
        for layer in self.quant_linears:
            layer.post_init(tuning_params, shared_cache)
        return self

    def set_tuning_param(self, tuning_params: MarlinTuningParams) -> "MarlinQuantLinearMaker":
        for layer in self.quant_linears:
            layer._matrix().set_tuning_params(tuning_params)
        return self

    def merge(self, linears: list[MarlinQuantLinear]) -> MarlinQuantLinear:
        """One layer over the given layers' output columns side by side (the merged q/k/v
        and gate/up of real_loader_marlin.py:65-79); the inputs leave the maker."""
        if not linears:
            raise ValueError("cannot merge an empty list of Marlin linears")
        head = linears[0]
        for attr, what in (("infeatures", "in_features"), ("group_size", "group_size"),
                           ("use_act_order", "act-order mode")):
            if any(getattr(l, attr) != getattr(head, attr) for l in linears):
                raise ValueError(f"merged Marlin linears must share {what}")
        if any(not torch.equal(l.g_idx, head.g_idx) for l in linears[1:]):
            raise ValueError("merged Marlin linears must share g_idx")
        merged = self.make_linear(head.infeatures, sum(l.outfeatures for l in linears), False)
        merged.qweight = torch.cat([l.qweight for l in linears], dim=1).contiguous()
        merged.qzeros = torch.cat([l.qzeros for l in linears], dim=1).contiguous()
        merged.scales = torch.cat([l.scales for l in linears], dim=1).contiguous()
        merged.g_idx = head.g_idx
        for l in linears:
            self.quant_linears.remove(l)
        return merged
