"""The tcgen05 GEMM's CTA-pair variant (cta_group::2, W4A16_TC_PAIR=1) against the
oracle and against the single-CTA kernel. The switch is read once per process, so the
pair kernel runs in a child process."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, sys
import numpy as np, torch
sys.path.insert(0, sys.argv[1])
from drofell_for_revision_b200 import _capi, synthetic
from oracle import w4a16_oracle as orc
out = {}
# even and odd column-tile counts (a pair's second CTA past N), act-order, bf16, M edges
for K, N, g, act, M, dt in [(1024, 1024, 128, False, 512, "fp16"), (2048, 384, 64, False, 300, "fp16"),
                            (1024, 1536, 128, True, 700, "fp16"), (512, 640, 32, False, 257, "bf16")]:
    layer = synthetic.make_layer(K, N, g, act_order=act, seed=K + N)
    h = _capi.Handle(layer.qweight.cuda(), layer.qzeros.cuda(), layer.scales.cuda(),
                     layer.g_idx if act else None, 0)
    dtype = torch.bfloat16 if dt == "bf16" else torch.float16
    x = synthetic.make_activations(M, K, seed=M, dtype=dtype)
    y = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
    h.gemm(x.cuda(), y, _capi.PATH_TC)
    torch.cuda.synchronize()
    xin = x.view(torch.int16).numpy().view(np.uint16) if dt == "bf16" else x.numpy()
    ref = orc.c_linear(xin, layer.qweight.numpy(), layer.qzeros.numpy(), layer.scales.numpy(),
                       layer.g_idx.numpy() if act else None, g, dtype=dt, threads=8)
    out[f"{K}x{N}_{M}_{dt}"] = {"err": float(orc.rel_err(y.float().cpu().numpy(), ref)),
                                "nan": bool(torch.isnan(y).any()), "dev_err": h.device_error()}
    np.save(sys.argv[2] + f"/{K}x{N}_{M}_{dt}.npy", y.float().cpu().numpy())
print(json.dumps(out))
"""


def _run(tmp, pair):
    env = dict(os.environ, W4A16_TC_PAIR="1" if pair else "0")
    res = subprocess.run([sys.executable, "-c", CHILD, ROOT, str(tmp)], env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    return json.loads(res.stdout.strip().splitlines()[-1])


def test_cta_pair_gemm_matches_oracle_and_single_cta(tmp_path):
    import numpy as np
    (tmp_path / "pair").mkdir()
    (tmp_path / "single").mkdir()
    pair = _run(tmp_path / "pair", True)
    single = _run(tmp_path / "single", False)
    for key, r in pair.items():
        tol = 8e-3 if key.endswith("bf16") else 2e-3
        assert not r["nan"] and r["dev_err"] == 0, (key, r)
        assert r["err"] < tol, (key, r["err"])
        a = np.load(tmp_path / "pair" / f"{key}.npy")
        b = np.load(tmp_path / "single" / f"{key}.npy")
        assert np.max(np.abs(a - b)) <= tol * max(1e-6, float(np.max(np.abs(b)))), key
