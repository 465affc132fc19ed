"""N-column-sharded W4A16 linear across the GPUs of one node.

Rank r of P owns output columns [r*N/P, (r+1)*N/P): its slice of qweight
[K/8, N/P], qzeros [G, N/(8P)] and scales [G, N/P]; g_idx is replicated. X is
replicated, so there is no input collective. Each rank computes Y_r [M, N/P] with
the local kernels and the slices are all-gathered into [M, N]:
  * with a PeerGather, for M up to the module's max_m: inside the kernel, which
    writes its columns into every rank's output over NVLink (w4a16_gemm_gather:
    the GEMV at decode sizes, the tcgen05 GEMM's epilogue above);
  * otherwise one NCCL all-gather of [P, M, N/P] and a permute (a view-only reshape
    when M == 1).

The reference has no tensor parallelism (its multi-GPU mode is a layer pipeline
over TCP, exps/infer_scale/README.md); this is the column split the quantized
linear admits because output columns are independent.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional

import torch
import torch.distributed as dist
from torch import nn

from ._capi import torch_fast_path


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


class PeerGather:
    """Peer-memory all-gather group of the ranks of ``group`` (one process per GPU).

    Wraps the C ABI's w4a16_comm: every rank's epoch flags are mapped into every other
    rank with CUDA IPC (handles exchanged with all_gather_object), and output buffers
    are registered the same way, so w4a16_gemm_gather can write every rank's full
    output over NVLink from inside the GEMV or GEMM kernel. Constructor and ``register`` are
    collective: every rank calls them in the same order.
    """

    def __init__(self, rank: int, world: int, device: torch.device, group=None):
        from . import _capi
        self.rank, self.world, self.device, self.group = rank, world, device, group
        self.comm = _capi.Comm(rank, world, device.index if device.index is not None else 0)
        handles = [None] * world
        dist.all_gather_object(handles, self.comm.flags_handle(), group=group)
        for p in range(world):
            if p != rank:
                self.comm.set_peer_flags(p, handles[p])

    def register(self, t: torch.Tensor) -> list:
        """Every rank's ``t`` as addressable from this process (rank order)."""
        from . import _capi
        handles = [None] * self.world
        dist.all_gather_object(handles, _capi.ipc_export(t), group=self.group)
        return [t.data_ptr() if p == self.rank else self.comm.open(handles[p]) for p in range(self.world)]

    def close(self) -> None:
        self.comm.close()


class GatherTimeout(RuntimeError):
    """A fused all-gather gave up waiting for another rank (its output is incomplete)."""


class ShardedQuantLinear(nn.Module):
    """Column-parallel wrapper: a local linear over this rank's columns + all-gather.

    ``local`` is any module mapping [M, K] -> [M, N/P]; :func:`from_packed` builds
    the B200 ``QuantLinear`` for it. ``local_forward`` may replace the module call
    (tests use it to run the path on CPU ranks).

    Failure detection on the fused path: a rank that never arrives makes the
    completion kernel's bounded wait give up and set the handle's device error word;
    the output then holds stale columns of that rank. The forward does not read the
    word (that would synchronise the stream and break graph capture). Instead:
      * ``check_gather()`` reads it and raises :class:`GatherTimeout` if a wait gave
        up since the last check; serving loops call it between steps;
      * ``check_every=n`` makes every n-th fused forward call it (eager use only).
    """

    def __init__(self, local: Optional[nn.Module], N: int, rank: int, world: int, group=None,
                 local_forward: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                 peer: Optional[PeerGather] = None, max_m: int = 16, check_every: int = 0):
        super().__init__()
        self.check_every = check_every
        self._fused_calls = 0
        self.local = local
        self.N = N
        self.rank = rank
        self.world = world
        self.group = group
        self._local_forward = local_forward
        # fused path (fp16, M <= max_m rows; 2 x max_m x N fp16 of buffers): this
        # module's full output lives in buffers every rank writes into, used in turns: a
        # forward's result is a view of one, rewritten two forwards later. Other ranks
        # write the next turn's buffer only after this rank has signalled the forward in
        # between, i.e. after its stream has run the consumers it ordered before that
        # forward.
        self.peer = peer
        self.max_m = max_m
        self._y_full = None
        self._y_ptrs = None
        self._turn = 0
        if peer is not None and world > 1:
            if local is None or getattr(local, "bias", None) is not None:
                raise ValueError("the fused gather needs a bias-free QuantLinear")
            self._y_full = [torch.empty((max_m, N), dtype=torch.float16, device=peer.device) for _ in range(2)]
            self._y_ptrs = [peer.register(b) for b in self._y_full]
            # the same pointers as host arrays, built once: the C++ forward takes their address
            self._y_arrs = [(ctypes.c_void_p * world)(*ptrs) for ptrs in self._y_ptrs]

    @classmethod
    def from_packed(cls, qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, g_idx: torch.Tensor,
                    group_size: int, act_order: bool, rank: int, world: int, device: torch.device, group=None,
                    tuning_params=None, cache=None, peer: Optional[PeerGather] = None,
                    max_m: int = 16) -> "ShardedQuantLinear":
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
        return cls(lin, N, rank, world, group, peer=peer, max_m=max_m)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.world == 1 and self._local_forward is None:
            return self.local(x)  # one rank: the local linear is the whole layer
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        if (self._y_full is not None and x2.dtype == torch.float16 and 0 < x2.shape[0] <= self.max_m
                and not x2.requires_grad):
            # GEMV / GEMM with the all-gather fused in (w4a16_gemm_gather): no NCCL
            per = self.N // self.world
            t = self._turn
            self._turn ^= 1
            h = self.local.q4_matrix._h
            fast = torch_fast_path()
            if fast is not None:  # one C++ call (the same C ABI), as QuantLinear's forward
                fast.gemm_gather(h.ptr, self.peer.comm.ptr, x2.contiguous(), ctypes.addressof(self._y_arrs[t]),
                                 self.N, self.rank * per)
            else:
                h.gemm_gather(x2.contiguous(), self.peer.comm, self._y_ptrs[t], self.N, self.rank * per)
            self._fused_calls += 1
            if self.check_every > 0 and self._fused_calls % self.check_every == 0:
                self.check_gather()
            return self._y_full[t][:x2.shape[0]].view(*lead, self.N)
        y_local = self._local_forward(x2) if self._local_forward is not None else self.local(x2)
        y = gather_columns(y_local.reshape(-1, self.N // self.world), self.world, self.group)
        return y.view(*lead, self.N)

    def check_gather(self) -> None:
        """Raise :class:`GatherTimeout` if a fused all-gather of this module gave up
        waiting for a rank since the last check (reads and clears the handle's device
        error word; synchronises the current stream)."""
        if self._y_full is None:
            return
        err = self.local.q4_matrix._h.device_error()
        if err != 0:
            raise GatherTimeout(f"rank {self.rank}: a fused all-gather gave up waiting for another rank "
                                f"(device error {err}); the last outputs are incomplete")
