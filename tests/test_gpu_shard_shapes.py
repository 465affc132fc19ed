"""The per-rank work of the column-sharded runs, on one GPU: every merged projection of
the Llama-2-7B and Llama-2-70B layers cut to the N/P columns one of P = 2, 4 or 8 ranks
holds (what `bench.py --gpus P` runs on each rank before the gather), at the decode and
prefill sizes the bench times. Some shards end in a partial 128-column tile
(22016 / 8 = 2752 columns).

Checks per case: 8-aligned column blocks against the oracle, the whole
output against a torch fp32 GEMM on the bit-exact dequantized weight (the path's own
bound), and a clean device error word.
"""
import numpy as np
import pytest
import torch

from drofell_for_revision_b200 import _capi, synthetic
from oracle import w4a16_oracle as orc

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
TOL = 1e-2
TOL_GEMV = 4e-3
TOL_TC = 2e-3

MERGED_7B = [(4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096)]   # qkv, o, gate_up, down
MERGED_70B = [(8192, 10240), (8192, 8192), (8192, 57344), (28672, 8192)]

CASES = [(K, N, P, (1, 8, 2048)) for K, N in MERGED_7B for P in (2, 4, 8)]
CASES += [(K, N, P, (1, 16, 128)) for K, N in MERGED_70B for P in (2, 4, 8)]


@pytest.mark.parametrize("K,N,P,Ms", CASES, ids=[f"{K}x{N}/{P}" for K, N, P, _ in CASES])
def test_rank_shard_matches_oracle(K, N, P, Ms):
    assert N % P == 0 and (N // P) % 8 == 0  # qzeros packs 8 columns per word
    n = N // P
    layer = synthetic.make_layer(K, n, 128, seed=K + n + P)
    h = _capi.Handle(layer.qweight.to(DEV), layer.qzeros.to(DEV), layer.scales.to(DEV), None, 0)
    w = torch.empty((K, n), dtype=torch.float16, device=DEV)
    h.dequant(w)
    torch.backends.cuda.matmul.allow_tf32 = False
    rng = np.random.default_rng(K + n)
    starts = np.sort(rng.choice(n // 8, size=min(6, n // 8), replace=False)) * 8
    starts[-1] = n - 8  # the last columns: a partial tile where n % 128 != 0
    cols = np.unique(np.concatenate([np.arange(s, s + 8) for s in starts]))
    for M in Ms:
        x = synthetic.make_activations(M, K, seed=M + P)
        xd = x.to(DEV)
        y = torch.full((M, n), float("nan"), dtype=torch.float16, device=DEV)
        h.gemm(xd, y)
        torch.cuda.synchronize()
        qw = layer.qweight[:, cols].numpy()
        qz = layer.qzeros[:, sorted(set(int(c) // 8 for c in cols))].numpy()
        ref = orc.w4a16_linear_ref(x.numpy(), qw, qz, layer.scales[:, cols].numpy(), None, 128)
        assert orc.rel_err(y[:, cols].float().cpu().numpy(), ref) < TOL, M
        yref = (xd.float() @ w.float()).cpu().numpy()
        assert orc.rel_err(y.float().cpu().numpy(), yref) < (TOL_GEMV if M <= 16 else TOL_TC), M
    assert h.device_error() == 0
    h.close()
