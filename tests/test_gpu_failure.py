"""Failure detection on the GPU without a fault: a bounded device-side wait on
a barrier that nothing completes gives up, the host reads the error status,
and the context keeps working."""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(cuda_ops):
    from triton_ssm_b200 import _lib
    lib = _lib.load_library()
    cuda_ops.check_device_status()          # start from a clean status word
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.time()
    assert lib.tssm_selftest_wait_timeout(100_000_000, stream) == 0
    with pytest.raises(TimeoutError):
        cuda_ops.check_device_status()
    assert time.time() - t0 < 10
    # the status word was cleared and the context still runs kernels
    cuda_ops.check_device_status()
    x = torch.randn(2, 64, 8, device="cuda")
    y, h = cuda_ops.ssm_forward(x, torch.full_like(x, 0.5), x, x, torch.zeros(8, device="cuda"))
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
