"""A gather group whose other rank never arrives, on one GPU.

Rank 1 of a 2-rank group is a flags buffer that nothing writes. The signal kernel
after the GEMV gives up its bounded wait, records the gather timeout (128) in the
handle's device error word, and the CUDA context stays usable. No fault, trap or
hang is involved: the wait's iteration limit ends it.
"""
import ctypes

import pytest
import torch

from drofell_for_revision_b200 import _capi, synthetic
from oracle import w4a16_oracle as orc

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
ERR_GATHER_TIMEOUT = 128  # kErrGatherTimeout in w4a16_gather.cuh


def test_wait_for_a_rank_that_never_arrives_gives_up():
    K, N = 1024, 512
    layer = synthetic.make_layer(K, N, 128, seed=5)
    h = _capi.Handle(layer.qweight.to(DEV), layer.qzeros.to(DEV), layer.scales.to(DEV), None, 0)
    comm = _capi.Comm(0, 2, 0)
    try:
        dead_flags = torch.zeros(2, dtype=torch.int32, device=DEV)  # rank 1's flags: never raised
        _capi.check(_capi.lib().w4a16_comm_set_peer_flags(ctypes.c_void_p(comm.ptr), 1,
                                                          ctypes.c_void_p(dead_flags.data_ptr())))
        y0 = torch.zeros((1, 2 * N), dtype=torch.float16, device=DEV)  # this rank's full Y
        y1 = torch.zeros((1, 2 * N), dtype=torch.float16, device=DEV)  # "rank 1's" Y, here local
        x = synthetic.make_activations(1, K, seed=1).to(DEV)
        h.gemm_gather(x, comm, [y0.data_ptr(), y1.data_ptr()], 2 * N, 0)
        torch.cuda.synchronize()
        assert h.device_error() == ERR_GATHER_TIMEOUT
        # this rank's columns reached both outputs before the wait
        ref = orc.w4a16_linear_ref(x.cpu().numpy(), layer.qweight.numpy(), layer.qzeros.numpy(),
                                   layer.scales.numpy(), None, layer.group_size)
        for y in (y0, y1):
            assert orc.rel_err(y[:, :N].float().cpu().numpy(), ref) < 4e-3
        assert int(dead_flags[0].item()) == 1  # this rank raised its epoch in rank 1's flags
        # the context is still usable and the error word was cleared by the read above
        y = torch.empty((1, N), dtype=torch.float16, device=DEV)
        h.gemm(x, y)
        torch.cuda.synchronize()
        assert orc.rel_err(y.float().cpu().numpy(), ref) < 4e-3
        assert h.device_error() == 0
    finally:
        comm.close()


class _OneGpuPeer:
    """A PeerGather stand-in for a 2-rank group on one GPU: rank 1 is a flags buffer
    that nothing writes and an output buffer that nothing reads."""

    def __init__(self):
        self.device = DEV
        self.comm = _capi.Comm(0, 2, 0)
        self.dead_flags = torch.zeros(2, dtype=torch.int32, device=DEV)
        _capi.check(_capi.lib().w4a16_comm_set_peer_flags(ctypes.c_void_p(self.comm.ptr), 1,
                                                          ctypes.c_void_p(self.dead_flags.data_ptr())))
        self._other = []

    def register(self, t):
        o = torch.zeros_like(t)
        self._other.append(o)
        return [t.data_ptr(), o.data_ptr()]

    def close(self):
        self.comm.close()


@pytest.mark.parametrize("check_every", [0, 1])
def test_sharded_module_reports_the_timeout(check_every):
    """ShardedQuantLinear surfaces the device error word as GatherTimeout: through
    check_gather() between steps, or inside the forward with check_every."""
    from drofell_for_revision_b200 import exllama, real_quant, sharded
    K, N = 1024, 512
    layer = synthetic.make_layer(K, N, 128, seed=6)
    lin = real_quant.QuantLinear(128, K, N, False, False)
    lin.qweight.copy_(layer.qweight)
    lin.qzeros.copy_(layer.qzeros)
    lin.scales.copy_(layer.scales)
    lin = lin.to(DEV)
    lin.post_init(exllama.TuningParams(), exllama.CacheV2(DEV))
    peer = _OneGpuPeer()
    try:
        mod = sharded.ShardedQuantLinear(lin, 2 * N, 0, 2, peer=peer, max_m=4, check_every=check_every)
        x = synthetic.make_activations(1, K, seed=2).to(DEV)
        if check_every:
            with pytest.raises(sharded.GatherTimeout):
                mod(x)
        else:
            mod(x)
            with pytest.raises(sharded.GatherTimeout):
                mod.check_gather()
        mod.check_gather()  # the word was cleared by the read that raised
    finally:
        peer.close()


@pytest.mark.parametrize("M", [8, 64])  # mma.sync GEMV, tcgen05 GEMM: 16-byte row pieces
def test_gather_rejects_outputs_off_16_byte_alignment(M):
    # checked on the host before any launch: a rank's Y that the kernels would store
    # 16-byte pieces into must be 16-byte aligned
    K, N = 1024, 512
    layer = synthetic.make_layer(K, N, 128, seed=5)
    h = _capi.Handle(layer.qweight.to(DEV), layer.qzeros.to(DEV), layer.scales.to(DEV), None, 0)
    comm = _capi.Comm(0, 2, 0)
    try:
        flags = torch.zeros(2, dtype=torch.int32, device=DEV)
        _capi.check(_capi.lib().w4a16_comm_set_peer_flags(ctypes.c_void_p(comm.ptr), 1,
                                                          ctypes.c_void_p(flags.data_ptr())))
        y0 = torch.zeros((M, 2 * N), dtype=torch.float16, device=DEV)
        y1 = torch.zeros((M, 2 * N + 8), dtype=torch.float16, device=DEV)
        x = synthetic.make_activations(M, K, seed=1).to(DEV)
        with pytest.raises(_capi.W4A16Error) as ei:
            h.gemm_gather(x, comm, [y0.data_ptr(), y1.data_ptr() + 2], 2 * N, 0)
        assert ei.value.code == _capi.W4A16_ERR_INVALID
        assert "16-byte aligned" in str(ei.value)
        torch.cuda.synchronize()
        assert h.device_error() == 0  # nothing was launched
    finally:
        comm.close()
        h.close()
