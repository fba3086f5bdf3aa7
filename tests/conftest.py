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


# Parity margins recorded by parity(): printed at the end of the session.
_MARGINS = []


def err_stats(out, ref):
    """Max-normalised error of one tensor: (max|out - ref| / max|ref|, the
    per-element 99th percentile of |out - ref| / max|ref|).  Computed on
    out's device."""
    out = out.detach()
    dev = out.device
    ref = ref.detach().to(dev).float()
    d = (out.float() - ref).abs().flatten()
    den = ref.abs().max().item() if ref.numel() else 0.0
    if d.numel() == 0:
        return 0.0, 0.0
    num = d.max().item()
    k = max(1, int(0.99 * d.numel()))
    p99 = d.kthvalue(k).values.item() if d.numel() <= (1 << 27) else \
        d[torch.randint(0, d.numel(), (1 << 24,), device=dev)].kthvalue(int(0.99 * (1 << 24))).values.item()
    if den > 0:
        return num / den, p99 / den
    return num, p99


def rel_err(out, ref):
    """max|out - ref| / max|ref| (the parity bar's measure)."""
    return err_stats(out, ref)[0]


def parity(name, out, ref, tol):
    """Check one config-level tensor against its bar and record the margin
    (max-normalised error and its per-element p99) for the session summary."""
    m, p99 = err_stats(out, ref)
    _MARGINS.append((name, m, p99, tol))
    assert m < tol, "%s: max-normalised error %.3e >= %.1e (p99 %.3e)" % (name, m, tol, p99)
    return m


def pytest_terminal_summary(terminalreporter):
    if not _MARGINS:
        return
    tr = terminalreporter
    tr.section("parity margins (max|d|/max|ref| and its per-element p99, against the bar)")
    for name, m, p99, tol in _MARGINS:
        tr.write_line("%-58s max %.2e  p99 %.2e  bar %.0e  (%.1f%% of bar)" % (name, m, p99, tol, 100 * m / tol))


@pytest.fixture(scope="session")
def cuda_ops():
    """The built CUDA extension; GPU tests fail loudly if it is missing."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import triton_ssm_b200 as ts
    ts.load_library()
    return ts
