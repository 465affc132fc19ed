"""The decoder-layer blocks around the projections, through the C ABI and the
reference-named Python entry points, against the oracle.

  * w4a16_rms_norm / w4a16_silu_mul: the reference's rms_norm_cuda and silu_mul_kernel
    (fuse_v2/rms_norm.cu:27-131, fuse_v2/q_mlp.cu:12-85);
  * w4a16_mlp_forward / mlp_forward_v2: RMSNorm -> gate, up -> silu * mul -> down
    (fuse_v2/q_mlp.cu:96-133), two launches at decode sizes, the unfused chain otherwise;
  * w4a16_qkv_forward / attention_forward_qkv_stage_v2: RMSNorm -> q, k, v
    (fuse_v2/q_attn.cu:23-54), one launch at decode sizes.
Tolerances: RMSNorm and silu * mul within 2 fp16 ulps of the fp32 restatement (the
reference's own fp16 silu is looser); the blocks max|Y - Y_ref| / max|Y_ref| <= 1e-2,
the north-star bound, and fused against unfused <= 5e-3.
"""
import numpy as np
import pytest
import torch

from drofell_for_revision_b200 import _capi, exllama, synthetic
from oracle import w4a16_oracle as orc

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
TOL = 1e-2
EPS = 1e-5


def _layer(K, N, act=False, seed=0, g=128):
    return synthetic.make_layer(K, N, g, act_order=act, seed=seed)


def _h(layer):
    return _capi.Handle(layer.qweight.to(DEV), layer.qzeros.to(DEV), layer.scales.to(DEV),
                        layer.g_idx if layer.act_order else None, 0)


def _args(layer):
    return (layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(),
            layer.g_idx.numpy() if layer.act_order else None, layer.group_size)


def _norm_w(K, seed):
    return (1.0 + 0.1 * torch.randn(K, generator=torch.Generator().manual_seed(seed))).half()


def _ulps(a, b):
    a16 = np.asarray(a, dtype=np.float16).astype(np.float32)
    b16 = np.asarray(b, dtype=np.float16).astype(np.float32)
    spacing = np.spacing(np.maximum(np.abs(a16), np.abs(b16)).astype(np.float16)).astype(np.float32)
    return float(np.max(np.abs(a16 - b16) / np.maximum(spacing, 2.0 ** -24)))


@pytest.mark.parametrize("M,K", [(1, 4096), (3, 5120), (64, 8192), (5, 64)])
def test_rms_norm(M, K):
    x = synthetic.make_activations(M, K, seed=K + M) * 3
    w = _norm_w(K, 1)
    out = torch.empty((M, K), dtype=torch.float16, device=DEV)
    _capi.rms_norm(x.to(DEV), w.to(DEV), EPS, out)
    torch.cuda.synchronize()
    assert _ulps(out.cpu().numpy(), orc.rms_norm_ref(x.numpy(), w.numpy(), EPS)) <= 2


@pytest.mark.parametrize("M,N", [(1, 11008), (7, 13824), (1, 64)])
def test_silu_mul(M, N):
    g = synthetic.make_activations(M, N, seed=N) * 4
    u = synthetic.make_activations(M, N, seed=N + 1)
    out = torch.empty((M, N), dtype=torch.float16, device=DEV)
    _capi.silu_mul(g.to(DEV), u.to(DEV), out)
    torch.cuda.synchronize()
    assert _ulps(out.cpu().numpy(), orc.silu_mul_ref(g.numpy(), u.numpy())) <= 2


def _mlp(K, I, act, seed, g=128):
    return _layer(K, I, act, seed, g), _layer(K, I, act, seed + 1, g), _layer(I, K, act, seed + 2, g)


def _run_mlp(hs, x, w, M, K, I):
    y = torch.full((M, K), float("nan"), dtype=torch.float16, device=DEV)
    r = torch.empty((M, K), dtype=torch.float16, device=DEV)
    g = torch.empty((M, I), dtype=torch.float16, device=DEV)
    u = torch.empty((M, I), dtype=torch.float16, device=DEV)
    _capi.mlp_forward(*hs, w, EPS, x, y, r, g, u)
    torch.cuda.synchronize()
    return y, r


# 7B / 13B MLP shapes, a small one with I % 128 != 0 (group size 32), and act-order
# (the unfused chain)
@pytest.mark.parametrize("K,I,act,g", [(4096, 11008, False, 128), (5120, 13824, False, 128), (512, 800, False, 32),
                                       (1024, 2048, True, 128)])
@pytest.mark.parametrize("M", [1, 2, 5, 40])
def test_mlp_forward(K, I, act, g, M, monkeypatch):
    layers = _mlp(K, I, act, seed=K + I, g=g)
    hs = [_h(l) for l in layers]
    x = synthetic.make_activations(M, K, seed=M)
    w = _norm_w(K, 2)
    xd, wd = x.to(DEV), w.to(DEV)
    y, r = _run_mlp(hs, xd, wd, M, K, I)
    fused = M <= 2 and not act
    assert (_capi.lib().w4a16_mlp_workspace_size(hs[0].ptr, hs[1].ptr, hs[2].ptr, M, 0) == 0) or not fused
    ref = orc.mlp_ref(x.numpy(), w.numpy(), EPS, *[_args(l) for l in layers])
    assert orc.rel_err(y.float().cpu().numpy(), ref) < TOL
    # the RMSNorm output is the standalone kernel's, bit for bit
    r2 = torch.empty_like(r)
    _capi.rms_norm(xd, wd, EPS, r2)
    torch.cuda.synchronize()
    assert torch.equal(r, r2)
    if fused:  # the same block through the unfused chain
        monkeypatch.setenv("W4A16_FUSE", "0")
        y2, _ = _run_mlp(hs, xd, wd, M, K, I)
        assert orc.rel_err(y.float().cpu().numpy(), y2.float().cpu().numpy()) < 5e-3
    for h in hs:
        assert h.device_error() == 0


@pytest.mark.parametrize("K,Nq,Nkv,act", [(4096, 4096, 4096, False), (8192, 8192, 1024, False),
                                          (1024, 1024, 256, True)])
@pytest.mark.parametrize("M", [1, 2, 3, 100])
def test_qkv_forward(K, Nq, Nkv, act, M, monkeypatch):
    lq, lk, lv = _layer(K, Nq, act, 11), _layer(K, Nkv, act, 12), _layer(K, Nkv, act, 13)
    hs = [_h(l) for l in (lq, lk, lv)]
    x = synthetic.make_activations(M, K, seed=M + 7)
    w = _norm_w(K, 3)
    outs = [torch.full((M, n), float("nan"), dtype=torch.float16, device=DEV) for n in (Nq, Nkv, Nkv)]
    r = torch.empty((M, K), dtype=torch.float16, device=DEV)
    _capi.qkv_forward(*hs, w.to(DEV), EPS, x.to(DEV), r, *outs)
    torch.cuda.synchronize()
    rr, *refs = orc.qkv_ref(x.numpy(), w.numpy(), EPS, _args(lq), _args(lk), _args(lv))
    assert _ulps(r.cpu().numpy(), rr) <= 2
    for o, ref in zip(outs, refs):
        assert orc.rel_err(o.float().cpu().numpy(), ref) < TOL


def test_fused_blocks_in_a_cuda_graph():
    K, I = 4096, 11008
    layers = _mlp(K, I, False, seed=5)
    hs = [_h(l) for l in layers]
    x = synthetic.make_activations(1, K, seed=9).to(DEV)
    w = _norm_w(K, 4).to(DEV)
    y = torch.empty((1, K), dtype=torch.float16, device=DEV)
    bufs = [torch.empty((1, K), dtype=torch.float16, device=DEV), torch.empty((1, I), dtype=torch.float16, device=DEV),
            torch.empty((1, I), dtype=torch.float16, device=DEV)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _capi.mlp_forward(*hs, w, EPS, x, y, *bufs)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        _capi.mlp_forward(*hs, w, EPS, x, y, *bufs)
    y.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    ref = orc.mlp_ref(x.cpu().numpy(), w.cpu().numpy(), EPS, *[_args(l) for l in layers])
    assert orc.rel_err(y.float().cpu().numpy(), ref) < TOL


def test_reference_named_entry_points():
    """mlp_forward_v2 / attention_forward_qkv_stage_v2 with the reference's arguments, on
    QuantLinear-built matrices (the q4 integers DecoderWrapFuse passes)."""
    from drofell_for_revision_b200 import real_quant
    K, I = 1024, 2816

    def ql(layer):
        m = real_quant.QuantLinear(128, layer.K, layer.N, False, False)
        m.qweight.copy_(layer.qweight)
        m.qzeros.copy_(layer.qzeros)
        m.scales.copy_(layer.scales)
        m = m.to(DEV)
        m.post_init(exllama.TuningParams(), exllama.CacheV2(DEV))
        return m

    lg, lu, ld = _mlp(K, I, False, seed=21)
    mg, mu, md = ql(lg), ql(lu), ql(ld)
    lq, lk, lv = _layer(K, K, False, 31), _layer(K, K, False, 32), _layer(K, K, False, 33)
    mq, mk, mv = ql(lq), ql(lk), ql(lv)
    bsz = 2
    x = synthetic.make_activations(bsz, K, seed=3).view(bsz, 1, K)
    w = _norm_w(K, 6)
    xd, wd = x.to(DEV), w.to(DEV)
    rms = torch.empty((bsz, K), dtype=torch.float16, device=DEV)
    q, k, v = (torch.empty((bsz, K), dtype=torch.float16, device=DEV) for _ in range(3))
    exllama.attention_forward_qkv_stage_v2_py(wd, EPS, mq.q4_matrix.cuda_q4, mk.q4_matrix.cuda_q4,
                                              mv.q4_matrix.cuda_q4, rms, q, k, v, None, xd, 128, 8, 50, 1, bsz)
    out = torch.empty((bsz, K), dtype=torch.float16, device=DEV)
    tg, tu = torch.empty((bsz, I), dtype=torch.float16, device=DEV), torch.empty((bsz, I), dtype=torch.float16, device=DEV)
    exllama.mlp_forward_v2_py(wd, EPS, mg.q4_matrix.cuda_q4, mu.q4_matrix.cuda_q4, md.q4_matrix.cuda_q4, rms, tg, tu,
                              None, xd.view(-1, K), out, 128, 8, 50)
    torch.cuda.synchronize()
    x2 = x.view(-1, K).numpy()
    _, rq, rk, rv = orc.qkv_ref(x2, w.numpy(), EPS, _args(lq), _args(lk), _args(lv))
    for o, ref in ((q, rq), (k, rk), (v, rv)):
        assert orc.rel_err(o.float().cpu().numpy(), ref) < TOL
    ref = orc.mlp_ref(x2, w.numpy(), EPS, _args(lg), _args(lu), _args(ld))
    assert orc.rel_err(out.float().cpu().numpy(), ref) < TOL
