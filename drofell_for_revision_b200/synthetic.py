"""Seeded synthetic GPTQ layers with the distributions the benchmark configs name.

qweight int32 [K/8, N] of uniform random words (8 uniform nibbles 0..15 along K);
qzeros int32 [G, N/8] likewise; scales fp16 = |N(0, 0.02)| + 1e-3; activations
fp16 ~ N(0, 1). Act-order: g_idx[k] = randperm(K)[k] // group_size, so every group
has exactly group_size members. Generated on the CPU with a torch.Generator so
CPU and GPU runs see identical inputs. The checkpoints the reference benchmarks
(split_qllm_models) are not available; these stand in for them.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

# Llama-2 projection shapes (in_features K, out_features N)
LLAMA2_7B = {
    "q_proj": (4096, 4096), "k_proj": (4096, 4096), "v_proj": (4096, 4096), "o_proj": (4096, 4096),
    "gate_proj": (4096, 11008), "up_proj": (4096, 11008), "down_proj": (11008, 4096),
}
LLAMA2_13B = {
    "q_proj": (5120, 5120), "k_proj": (5120, 5120), "v_proj": (5120, 5120), "o_proj": (5120, 5120),
    "gate_proj": (5120, 13824), "up_proj": (5120, 13824), "down_proj": (13824, 5120),
}
LLAMA2_70B = {
    "q_proj": (8192, 8192), "k_proj": (8192, 1024), "v_proj": (8192, 1024), "o_proj": (8192, 8192),
    "gate_proj": (8192, 28672), "up_proj": (8192, 28672), "down_proj": (28672, 8192),
}


@dataclass
class GPTQLayer:
    qweight: torch.Tensor
    qzeros: torch.Tensor
    scales: torch.Tensor
    g_idx: torch.Tensor
    group_size: int
    act_order: bool

    @property
    def K(self) -> int:
        return self.qweight.shape[0] * 8

    @property
    def N(self) -> int:
        return self.qweight.shape[1]

    def to(self, device) -> "GPTQLayer":
        return GPTQLayer(self.qweight.to(device), self.qzeros.to(device), self.scales.to(device),
                         self.g_idx.to(device), self.group_size, self.act_order)


def _rand_words(shape, gen: torch.Generator) -> torch.Tensor:
    return torch.randint(-2**31, 2**31, shape, generator=gen, dtype=torch.int64).to(torch.int32)


def make_layer(K: int, N: int, group_size: int = 128, act_order: bool = False, seed: int = 0,
               gen: Optional[torch.Generator] = None) -> GPTQLayer:
    gs = K if group_size == -1 else group_size
    if gen is None:
        gen = torch.Generator().manual_seed(seed)
    G = K // gs
    qweight = _rand_words((K // 8, N), gen)
    qzeros = _rand_words((G, N // 8), gen)
    scales = ((torch.randn((G, N), generator=gen) * 0.02).abs() + 1e-3).to(torch.float16)
    if act_order:
        g_idx = (torch.randperm(K, generator=gen) // gs).to(torch.int32)
    else:
        g_idx = (torch.arange(K) // gs).to(torch.int32)
    return GPTQLayer(qweight, qzeros, scales, g_idx, gs, act_order)


def make_activations(M: int, K: int, seed: int = 0, dtype: torch.dtype = torch.float16) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    return torch.randn((M, K), generator=gen).to(dtype)
