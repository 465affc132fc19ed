"""Generate golden vectors for the W4A16 dequant / linear from the reference's own code.

Run in a container that holds the reference tree (read-only) at REFERENCE_ROOT:

    python tests/golden/make_golden.py [REFERENCE_ROOT]

It imports ``operators.core.linear.real_quant.QuantLinear`` from the reference
(After-Revision-DROFELL/operators/core/linear/real_quant.py:10-102). The module's
CUDA-extension import is replaced by a stub (the extension is not built here),
and the AutoGPTQ shift table ``wf = arange(0, 32, 4)`` that
``get_reconstruct_weights`` expects (real_quant.py:72,81) is attached to each
instance, since the reference never defines it. ``get_reconstruct_weights`` then
runs unmodified and its fp16 output is stored as the golden dequant.

GEMM goldens are ``X.float() @ W.float()`` computed by torch on the CPU from that
same reference weight. bf16 goldens convert the reference fp16 weight the way the
reference's bf16 reconstruct kernel does (fp16 -> fp32 -> bf16 RNE,
cuda_extends/exllama/q4_matrix.cu:465-467).

The output, tests/golden/w4a16_golden.npz, is committed; tests read it without the
reference being present.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(root: str):
    sys.path.insert(0, os.path.join(root, "After-Revision-DROFELL"))
    stub = types.ModuleType("cuda_extends.exllama")
    for name in ["CacheV2", "ExllamaQ4ForwardOnlyLinearFunction", "ExllamaQ4LinearFunction",
                 "Q4MatrixV2", "TuningParams"]:
        setattr(stub, name, type(name, (), {}))
    import cuda_extends  # noqa: F401  (package __init__ only)
    sys.modules["cuda_extends.exllama"] = stub
    from operators.core.linear import real_quant
    return real_quant


def rand_i32(gen, shape):
    return torch.randint(-2**31, 2**31 - 1, shape, generator=gen, dtype=torch.int64).to(torch.int32)


def make_case(real_quant, name, K, N, group_size, act_order, seed, m_rows, mode="random"):
    gen = torch.Generator().manual_seed(seed)
    ql = real_quant.QuantLinear(group_size, K, N, False, act_order)
    ql.wf = torch.arange(0, 32, 4, dtype=torch.int32)
    gs = ql.group_size
    G = K // gs
    if mode == "random":
        ql.qweight.copy_(rand_i32(gen, ql.qweight.shape))
        ql.qzeros.copy_(rand_i32(gen, ql.qzeros.shape))
        ql.scales.copy_(((torch.randn(ql.scales.shape, generator=gen) * 0.02).abs() + 1e-3).half())
    elif mode == "extreme":
        # all-ones nibbles / zero nibble 0 and 15 / scales spanning subnormal..overflow, signs, zero
        ql.qweight.copy_(rand_i32(gen, ql.qweight.shape))
        ql.qweight[0].fill_(-1)             # every nibble 15
        ql.qweight[1].fill_(0)              # every nibble 0
        ql.qzeros.copy_(rand_i32(gen, ql.qzeros.shape))
        ql.qzeros[0].fill_(-1)              # zero nibble 15 -> z = 16
        if G > 1:
            ql.qzeros[1].fill_(0)           # zero nibble 0 -> z = 1
        pool = torch.tensor([0.0, -0.0, 6e-8, -6e-8, 1e-5, 3.05e-5, 0.5, -0.75, 1.0, 2.0,
                             1000.0, -2047.0, 4096.0, 4100.0, 65504.0, -65504.0], dtype=torch.float32)
        idx = torch.randint(0, pool.numel(), ql.scales.shape, generator=gen)
        ql.scales.copy_(pool[idx].half())
    else:
        raise ValueError(mode)
    if act_order:
        perm = torch.randperm(K, generator=gen)
        g_idx = (torch.arange(K) // gs)[torch.argsort(perm)].to(torch.int32)
        ql.g_idx.copy_(g_idx)
    w = ql.get_reconstruct_weights()
    assert w.dtype == torch.float16 and tuple(w.shape) == (K, N)
    x = torch.randn((m_rows, K), generator=gen).half()
    y = x.float() @ w.float()
    w_bf16 = w.float().to(torch.bfloat16)
    x_bf16 = x.float().to(torch.bfloat16)
    y_bf16 = x_bf16.float() @ w_bf16.float()
    out = {
        f"{name}/qweight": ql.qweight.numpy(),
        f"{name}/qzeros": ql.qzeros.numpy(),
        f"{name}/scales": ql.scales.numpy(),
        f"{name}/g_idx": ql.g_idx.numpy(),
        f"{name}/meta": np.array([K, N, gs, int(act_order)], dtype=np.int64),
        f"{name}/w_fp16": w.numpy(),
        f"{name}/w_bf16_bits": w_bf16.view(torch.int16).numpy().view(np.uint16),
        f"{name}/x_fp16": x.numpy(),
        f"{name}/y_fp32": y.numpy(),
        f"{name}/x_bf16_bits": x_bf16.view(torch.int16).numpy().view(np.uint16),
        f"{name}/y_bf16_fp32": y_bf16.numpy(),
    }
    return out


def make_uneven_case(real_quant, name, K, N, group_size, seed, m_rows):
    """Act-order table whose groups have unequal sizes (each a multiple of 8 rows)."""
    gen = torch.Generator().manual_seed(seed)
    ql = real_quant.QuantLinear(group_size, K, N, False, True)
    ql.wf = torch.arange(0, 32, 4, dtype=torch.int32)
    G = K // ql.group_size
    ql.qweight.copy_(rand_i32(gen, ql.qweight.shape))
    ql.qzeros.copy_(rand_i32(gen, ql.qzeros.shape))
    ql.scales.copy_(((torch.randn(ql.scales.shape, generator=gen) * 0.02).abs() + 1e-3).half())
    # blocks of 8 rows get a random group; then rows are shuffled
    blocks = torch.randint(0, G, (K // 8,), generator=gen)
    blocks[:G] = torch.arange(G)  # every group non-empty
    g = blocks.repeat_interleave(8)
    perm = torch.randperm(K, generator=gen)
    ql.g_idx.copy_(g[perm].to(torch.int32))
    w = ql.get_reconstruct_weights()
    x = torch.randn((m_rows, K), generator=gen).half()
    y = x.float() @ w.float()
    w_bf16 = w.float().to(torch.bfloat16)
    x_bf16 = x.float().to(torch.bfloat16)
    y_bf16 = x_bf16.float() @ w_bf16.float()
    return {
        f"{name}/qweight": ql.qweight.numpy(),
        f"{name}/qzeros": ql.qzeros.numpy(),
        f"{name}/scales": ql.scales.numpy(),
        f"{name}/g_idx": ql.g_idx.numpy(),
        f"{name}/meta": np.array([K, N, ql.group_size, 1], dtype=np.int64),
        f"{name}/w_fp16": w.numpy(),
        f"{name}/w_bf16_bits": w_bf16.view(torch.int16).numpy().view(np.uint16),
        f"{name}/x_fp16": x.numpy(),
        f"{name}/y_fp32": y.numpy(),
        f"{name}/x_bf16_bits": x_bf16.view(torch.int16).numpy().view(np.uint16),
        f"{name}/y_bf16_fp32": y_bf16.numpy(),
    }


CASES = [
    # name, K, N, group_size, act_order, seed, M, mode
    ("g32_k64_n32", 64, 32, 32, False, 1, 3, "random"),
    ("g128_k256_n64", 256, 64, 128, False, 2, 5, "random"),
    ("g64_k512_n96", 512, 96, 64, False, 3, 17, "random"),
    ("gfull_k128_n32", 128, 32, -1, False, 4, 2, "random"),
    ("act_g64_k256_n64", 256, 64, 64, True, 5, 4, "random"),
    ("act_g128_k512_n128", 512, 128, 128, True, 6, 33, "random"),
    ("extreme_g32_k128_n64", 128, 64, 32, False, 7, 2, "extreme"),
    ("g128_k1024_n64", 1024, 64, 128, False, 8, 65, "random"),
]


def main():
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DROFELL_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout root> "
                 "(or set DROFELL_REFERENCE_ROOT)")
    real_quant = load_reference(root)
    out = {}
    names = []
    for name, K, N, g, act, seed, m, mode in CASES:
        out.update(make_case(real_quant, name, K, N, g, act, seed, m, mode))
        names.append(name)
    out.update(make_uneven_case(real_quant, "act_uneven_g64_k256_n64", 256, 64, 64, 9, 3))
    names.append("act_uneven_g64_k256_n64")
    out["cases"] = np.array(names)
    path = os.path.join(HERE, "w4a16_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(names)} cases, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
