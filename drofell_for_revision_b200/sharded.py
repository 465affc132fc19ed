"""N-column-sharded W4A16 linear across the GPUs of one node.

Rank r of P owns output columns [r*N/P, (r+1)*N/P): its slice of qweight
[K/8, N/P], qzeros [G, N/(8P)] and scales [G, N/P]; g_idx is replicated. X is
replicated, so there is no input collective. Each rank computes Y_r [M, N/P] with
the local kernels, one all-gather (NCCL over NVLink/NVSwitch on GPUs) collects
[P, M, N/P], and a permute gives [M, N] (a view-only reshape when M == 1).

The reference has no tensor parallelism (its multi-GPU mode is a layer pipeline
over TCP, exps/infer_scale/README.md); this is the column split the quantized
linear admits because output columns are independent.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist
from torch import nn


def shard_bounds(N: int, rank: int, world: int) -> tuple[int, int]:
    if N % world != 0:
        raise ValueError(f"N={N} is not divisible by world size {world}")
    per = N // world
    if per % 32 != 0:
        raise ValueError(f"N/P={per} must be a multiple of 32 (the quantized linear's column granularity)")
    return rank * per, (rank + 1) * per


def shard_columns(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, rank: int, world: int):
    """Contiguous column slices of the packed tensors for ``rank``."""
    N = qweight.shape[1]
    n0, n1 = shard_bounds(N, rank, world)
    return (qweight[:, n0:n1].contiguous(), qzeros[:, n0 // 8:n1 // 8].contiguous(), scales[:, n0:n1].contiguous())


def gather_columns(y_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather [M, N/P] slices from every rank into [M, N] (rank-major columns)."""
    M, n_local = y_local.shape
    if world == 1:
        return y_local
    y_local = y_local.contiguous()
    backend = dist.get_backend(group)
    if backend == "nccl":
        gathered = torch.empty((world, M, n_local), dtype=y_local.dtype, device=y_local.device)
        dist.all_gather_into_tensor(gathered, y_local, group=group)
    else:
        parts = [torch.empty_like(y_local) for _ in range(world)]
        dist.all_gather(parts, y_local, group=group)
        gathered = torch.stack(parts, 0)
    if M == 1:
        return gathered.view(1, world * n_local)
    return gathered.permute(1, 0, 2).reshape(M, world * n_local)


class ShardedQuantLinear(nn.Module):
    """Column-parallel wrapper: a local linear over this rank's columns + all-gather.

    ``local`` is any module mapping [M, K] -> [M, N/P]; :func:`from_packed` builds
    the B200 ``QuantLinear`` for it. ``local_forward`` may replace the module call
    (tests use it to run the path on CPU ranks).
    """

    def __init__(self, local: Optional[nn.Module], N: int, rank: int, world: int, group=None,
                 local_forward: Optional[Callable[[torch.Tensor], torch.Tensor]] = None):
        super().__init__()
        self.local = local
        self.N = N
        self.rank = rank
        self.world = world
        self.group = group
        self._local_forward = local_forward

    @classmethod
    def from_packed(cls, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, g_idx: torch.Tensor,
                    group_size: int, act_order: bool, rank: int, world: int, device: torch.device, group=None,
                    tuning_params=None, cache=None) -> "ShardedQuantLinear":
        from .exllama import CacheV2, TuningParams
        from .real_quant import QuantLinear
        K, N = qweight.shape[0] * 8, qweight.shape[1]
        qw, qz, sc = shard_columns(qweight, qzeros, scales, rank, world)
        lin = QuantLinear(group_size, K, N // world, False, act_order)
        lin.qweight.copy_(qw)
        lin.qzeros.copy_(qz)
        lin.scales.copy_(sc)
        lin.g_idx.copy_(g_idx)
        lin = lin.to(device)
        cache = cache or CacheV2(device)
        lin.post_init(tuning_params or TuningParams(), cache)
        return cls(lin, N, rank, world, group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        y_local = self._local_forward(x2) if self._local_forward is not None else self.local(x2)
        y = gather_columns(y_local.reshape(-1, self.N // self.world), self.world, self.group)
        return y.view(*lead, self.N)
