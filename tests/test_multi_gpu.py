"""Column sharding with the all-gather fused into the kernel (peer memory over NVLink),
on 2 GPUs: the GEMV at decode sizes and the tcgen05 GEMM in both orientations (with and
without split-K) above. Outputs equal the NCCL path bit for bit and the unsharded kernel within the
kernels' tolerance, eagerly and inside CUDA graphs. Skipped on boxes with one GPU."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs 2 GPUs")


# the last shape's rank shard (1024 x 16384) runs the natural-orientation GEMM without a
# K split at M = 100 (its epilogue stores into the peers), with one at M = 40
SHAPES = [(4096, 4096, 128, False), (1024, 512, 64, True), (2048, 1024, 32, False), (1024, 32768, 128, False)]
MS = (1, 3, 8, 13, 40, 100, 300)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from drofell_for_revision_b200 import _capi, sharded, synthetic
        peer = sharded.PeerGather(rank, world, dev)
        results = {}
        for (K, N, g, act) in SHAPES:
            layer = synthetic.make_layer(K, N, g, act_order=act, seed=K + N)
            fused = sharded.ShardedQuantLinear.from_packed(layer.qweight, layer.qzeros, layer.scales, layer.g_idx, g,
                                                           act, rank, world, dev, peer=peer, max_m=320)
            plain = sharded.ShardedQuantLinear.from_packed(layer.qweight, layer.qzeros, layer.scales, layer.g_idx, g,
                                                           act, rank, world, dev)
            full = _capi.Handle(layer.qweight.to(dev), layer.qzeros.to(dev), layer.scales.to(dev),
                                layer.g_idx if act else None, rank)
            for M in MS:  # GEMV sizes, then the GEMM in both orientations, with and without a K split
                x = synthetic.make_activations(M, K, seed=M).to(dev)
                for rep in range(3):  # repeated calls: epochs advance
                    yf = fused(x).clone()
                yp = plain(x)
                yr = torch.empty((M, N), dtype=torch.float16, device=dev)
                full.gemm(x, yr)
                torch.cuda.synchronize()
                results[f"{K}x{N}_m{M}_fused"] = yf.float().cpu().numpy()
                results[f"{K}x{N}_m{M}_plain"] = yp.float().cpu().numpy()
                results[f"{K}x{N}_m{M}_full"] = yr.float().cpu().numpy()
            # inside a CUDA graph (flags and epochs live on the device)
            x = synthetic.make_activations(1, K, seed=99).to(dev)
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                fused(x)
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            gph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gph, stream=s):
                yg = fused(x)
            for _ in range(5):
                gph.replay()
            torch.cuda.synchronize()
            results[f"{K}x{N}_graph"] = yg.float().cpu().numpy()
            yr = torch.empty((1, N), dtype=torch.float16, device=dev)
            full.gemm(x, yr)
            torch.cuda.synchronize()
            results[f"{K}x{N}_graph_full"] = yr.float().cpu().numpy()
            del gph
            results[f"{K}x{N}_err"] = np.array([fused.local.q4_matrix._h.device_error()])
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), **results)
        dist.barrier()
        peer.close()
    finally:
        dist.destroy_process_group()


@needs_two
def test_fused_gather_on_two_gpus(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=False,
                             start_method="spawn")
    while not ctx.join(timeout=300):
        pass
    from drofell_for_revision_b200 import synthetic
    from oracle import w4a16_oracle as orc
    refs = {}
    for (K, N, g, act) in SHAPES:  # the oracle on the same seeded inputs as the workers
        layer = synthetic.make_layer(K, N, g, act_order=act, seed=K + N)
        args = (layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(),
                layer.g_idx.numpy() if act else None, layer.group_size)
        for M in MS:
            refs[f"{K}x{N}_m{M}"] = orc.w4a16_linear_ref(synthetic.make_activations(M, K, seed=M).numpy(), *args)
        refs[f"{K}x{N}"] = orc.w4a16_linear_ref(synthetic.make_activations(1, K, seed=99).numpy(), *args)
    for rank in range(world):
        r = np.load(tmp_path / f"r{rank}.npz")
        for key in r.files:
            if key.endswith("_fused"):
                base = key[:-len("_fused")]
                np.testing.assert_array_equal(r[key], r[base + "_plain"])
                assert orc.rel_err(r[key], r[base + "_full"]) < 4e-3, key
                assert orc.rel_err(r[key], refs[base]) < 4e-3, key  # and the oracle itself
            if key.endswith("_graph"):
                assert orc.rel_err(r[key], r[key + "_full"]) < 4e-3, key
                assert orc.rel_err(r[key], refs[key[:-len("_graph")]]) < 4e-3, key
            if key.endswith("_err"):
                assert int(r[key][0]) == 0, key
