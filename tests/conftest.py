import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# Parity bars (relative error = max|out - ref| / max|ref| per tensor).
TOL_FP32 = 1e-4          # fp32 inputs
TOL_BF16 = 2e-2          # bf16 inputs with fp32 state


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: torch.from_numpy(z[k].copy()) for k in z.files}


def rel_err(out, ref):
    out = out.detach().float().cpu()
    ref = ref.detach().float().cpu()
    den = ref.abs().max().item()
    num = (out - ref).abs().max().item()
    return num / den if den > 0 else num


@pytest.fixture(scope="session")
def cuda_ops():
    """The built CUDA extension; GPU tests fail loudly if it is missing."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import triton_ssm_b200 as ts
    ts.load_library()
    return ts
