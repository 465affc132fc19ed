"""Drop-in for the reference's quantized-linear operator.

Mirrors After-Revision-DROFELL/operators/core/linear/real.py:6-15 (``Linear`` /
``LinearMaker``) and operators/core/linear/real_quant.py:10-138 (``QuantLinear`` /
``QuantLinearMaker``): same constructor arguments, registered buffers (names,
dtypes, shapes), ``post_init`` / ``forward`` behaviour and asserts, so a
``state_dict`` saved for the reference loads unchanged. The forward runs the B200
W4A16 kernels through :mod:`drofell_for_revision_b200.exllama`.
"""
from __future__ import annotations

import math
from abc import ABC, abstractmethod
from typing import cast

import torch
from torch import nn

from . import flags
from ._capi import torch_fast_path
from .exllama import (CacheV2, ExllamaQ4ForwardOnlyLinearFunction, ExllamaQ4LinearFunction, Q4MatrixV2,
                      TuningParams)


class Linear(ABC, nn.Module):
    @abstractmethod
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError


class LinearMaker(ABC):
    @abstractmethod
    def make_linear(self, in_features: int, out_features: int, bias: bool) -> Linear:
        raise NotImplementedError


class QuantLinear(Linear):
    """GPTQ 4-bit linear (real_quant.py:10-49 layout)."""

    def __init__(self, group_size: int, in_features: int, out_features: int, bias: bool, use_act_order: bool):
        nn.Module.__init__(self)
        self.infeatures = in_features
        self.outfeatures = out_features
        self.use_act_order = use_act_order
        self.bits = 4
        self.group_size = group_size if group_size != -1 else in_features
        self.maxq = 2 ** self.bits - 1

        assert in_features % 32 == 0
        assert in_features % self.group_size == 0
        assert out_features % 32 == 0

        self.register_buffer("qweight", torch.zeros((in_features // 32 * self.bits, out_features), dtype=torch.int32))
        self.register_buffer("qzeros", torch.zeros((math.ceil(in_features / self.group_size),
                                                    out_features // 32 * self.bits), dtype=torch.int32))
        self.register_buffer("scales", torch.zeros((math.ceil(in_features / self.group_size), out_features),
                                                   dtype=torch.float16))
        self.register_buffer("g_idx", torch.tensor([i // self.group_size for i in range(in_features)],
                                                   dtype=torch.int32))
        if bias:
            self.register_buffer("bias", torch.zeros(out_features, dtype=torch.float16))
        else:
            self.bias = None

    def post_init(self, tunning_params: TuningParams, cache: CacheV2):
        assert self.qweight.device.type == "cuda"
        assert self.qweight.device.index is not None
        self.q4_matrix = Q4MatrixV2(
            self.qweight, self.qzeros, self.scales, self.infeatures, self.outfeatures,
            self.g_idx.cpu() if self.use_act_order else None, self.use_act_order,
            tuning_params=tunning_params, cache=cache)
        if flags.RECONSTRUCTE_WEIGTH_FLOAT16:
            self.q4_matrix.reconstruct_weight(dtype=torch.float16)
        if flags.RECONSTRUCTE_WEIGTH_BFLOAT16:
            self.q4_matrix.reconstruct_weight(dtype=torch.bfloat16)

    def get_reconstruct_weights(self) -> torch.Tensor:
        """Dense fp16 W [K, N] (the reference's torch dequant, real_quant.py:69-102,
        which raises there because ``self.wf`` is never defined); computed here by the
        bit-exact dequant kernel. Requires ``post_init``."""
        return self.q4_matrix.get_float16_weights_matrix_v2()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.requires_grad:
            return cast(torch.Tensor, ExllamaQ4LinearFunction.apply(x, self.q4_matrix, self.bias,
                                                                    flags.REUSE_RECONSTRUCT_CACHE_WHEN_GRAD))
        # nothing requires grad (the packed weights are buffers): the computation of
        # ExllamaQ4ForwardOnlyLinearFunction in one C++ call (torch fast path), or
        # through the ctypes binding where that extension was not built
        fast = torch_fast_path()
        if fast is not None:
            return fast.linear(self.q4_matrix.cuda_q4, x, self.bias)
        out = self.q4_matrix.matmul(x, None, None, False)
        if self.bias is not None:
            out += self.bias
        return out


class QuantLinearMaker(LinearMaker):
    """Builds the QuantLinear layers of one model and finishes them together
    (interface of real_quant.py:114-138): ``make_linear`` registers each layer,
    ``post_init`` binds every registered layer to the B200 kernels once, and
    ``set_tuning_param`` hands new parameters to every bound matrix."""

    def __init__(self, quantization_group_size: int, use_act_order: bool) -> None:
        self.quantization_group_size = quantization_group_size
        self.use_act_order = use_act_order
        self.quant_linears: list[QuantLinear] = []
        self.post_inited: bool = False

    def make_linear(self, in_features: int, out_features: int, bias: bool = False) -> QuantLinear:
        layer = QuantLinear(self.quantization_group_size, in_features, out_features, bias, self.use_act_order)
        self.quant_linears.append(layer)
        return layer

    def post_init(self, tunning_params: TuningParams, shared_cache: CacheV2) -> "QuantLinearMaker":
        assert not self.post_inited, "post_init runs once per maker"
        self.post_inited = True
        for layer in self.quant_linears:
            layer.post_init(tunning_params, shared_cache)
        return self

    def set_tuning_param(self, tuning_param: TuningParams) -> "QuantLinearMaker":
        for layer in self.quant_linears:
            layer.q4_matrix.set_tuning_params(tuning_param)
        return self
