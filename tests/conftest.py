import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    path = os.path.join(ROOT, "tests", "golden", "w4a16_golden.npz")
    data = np.load(path)
    cases = {}
    for name in data["cases"]:
        name = str(name)
        K, N, gs, act = (int(v) for v in data[f"{name}/meta"])
        cases[name] = {
            "K": K, "N": N, "group_size": gs, "act_order": bool(act),
            **{key: data[f"{name}/{key}"] for key in
               ["qweight", "qzeros", "scales", "g_idx", "w_fp16", "w_bf16_bits", "x_fp16", "y_fp32",
                "x_bf16_bits", "y_bf16_fp32"]},
        }
    return cases
