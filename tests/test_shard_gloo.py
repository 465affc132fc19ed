"""N-column sharding + all-gather on CPU ranks (gloo, world sizes 2, 4 and 8).

Each rank runs the oracle on its column slice as the local compute; the gathered
output must equal the unsharded oracle output bit for bit.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, M, K, N, act, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from drofell_for_revision_b200 import sharded, synthetic
        from oracle import w4a16_oracle as orc
        layer = synthetic.make_layer(K, N, 64, act_order=act, seed=11)
        x = synthetic.make_activations(M, K, seed=12)
        qw, qz, sc = sharded.shard_columns(layer.qweight, layer.qzeros, layer.scales, rank, world)
        gi = layer.g_idx.numpy() if act else None

        def local_forward(xx):
            y = orc.w4a16_linear_ref(xx.numpy(), qw.numpy(), qz.numpy(), sc.numpy(), gi, 64)
            return torch.from_numpy(y)

        mod = sharded.ShardedQuantLinear(None, N, rank, world, local_forward=local_forward)
        y = mod(x.view(1, M, K))
        assert y.shape == (1, M, N)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.view(M, N).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,M,act", [(2, 1, False), (2, 5, True), (4, 3, False), (8, 2, True)])
def test_sharded_equals_unsharded(tmp_path, world, M, act):
    K, N = 256, 256
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, M, K, N, act, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    from drofell_for_revision_b200 import synthetic
    from oracle import w4a16_oracle as orc
    layer = synthetic.make_layer(K, N, 64, act_order=act, seed=11)
    x = synthetic.make_activations(M, K, seed=12)
    ref = orc.w4a16_linear_ref(x.numpy(), layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(),
                               layer.g_idx.numpy() if act else None, 64)
    from drofell_for_revision_b200 import sharded
    gi = layer.g_idx.numpy() if act else None
    parts = []
    for r in range(world):
        qw, qz, sc = sharded.shard_columns(layer.qweight, layer.qzeros, layer.scales, r, world)
        parts.append(orc.w4a16_linear_ref(x.numpy(), qw.numpy(), qz.numpy(), sc.numpy(), gi, 64))
    expect = np.concatenate(parts, 1)
    for r in range(world):
        y = np.load(tmp_path / f"y{r}.npy")
        np.testing.assert_array_equal(y, expect)  # gather + permute is exact
        assert orc.rel_err(y, ref) < 1e-6          # and equals the unsharded layer
