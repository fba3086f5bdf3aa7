"""The entry point for callers that cannot allocate device memory at call time
(tssm_interp_ssm_static_scratch: scratch in a fixed array inside the library)
must give the same results as tssm_interp_ssm with a caller-provided
workspace, call after call.  This file is named to be collected last."""
import ctypes

import pytest
import torch

import oracle
from conftest import TOL_FP32, rel_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def _inputs(seed=21, Bt=4, T=300, Dm=64, N=16, Lq=500):
    g = torch.Generator().manual_seed(seed)
    V = torch.randn(Bt, T, Dm, generator=g)
    M = (torch.rand(Bt, T, Dm, generator=g) < 0.7).to(torch.uint8)
    tau = torch.cumsum(torch.empty(Bt, T).exponential_(1.0, generator=g), 1)
    A_log = torch.log(torch.arange(1, N + 1, dtype=torch.float32)).repeat(Dm, 1)
    B = torch.randn(Dm, N, generator=g) / N ** 0.5
    C = torch.randn(Dm, N, generator=g) / N ** 0.5
    D = torch.randn(Dm, generator=g)
    q = oracle.linspace_queries(tau, Lq)
    dt = (tau[:, -1] - tau[:, 0]) / (Lq - 1)
    return [t.to(dev).contiguous() for t in (V, M, tau, q, A_log, B, C, D, dt)]


def _call_static(lib, V, M, tau, q, A_log, B, C, D, dt, y, h, FTILE=128):
    P = ctypes.c_void_p
    Bt, T, Dm = V.shape
    N = A_log.shape[1]
    Lq = q.shape[1]
    st = lib.tssm_interp_ssm_static_scratch(
        P(V.data_ptr()), P(M.data_ptr()), P(tau.data_ptr()), P(q.data_ptr()), P(A_log.data_ptr()),
        P(B.data_ptr()), P(C.data_ptr()), P(D.data_ptr()), P(dt.data_ptr()), P(y.data_ptr()), P(h.data_ptr()),
        P(0), Bt, T, Dm, N, Lq, 10, FTILE, 3, P(torch.cuda.current_stream().cuda_stream))
    return st


def _check_against_workspace_entry(cuda_ops, lib, inputs, FTILE):
    V, M, tau, q, A_log, B, C, D, dt = inputs
    y_ref, h_ref = cuda_ops.fused_interp_ssm(V, M, tau, A_log, B, C, q=q, dt=dt, D=D, FTILE=FTILE,
                                             return_state=True)
    y = torch.full_like(y_ref, float("nan"))   # poisoned: every element must be written
    h = torch.full_like(h_ref, float("nan"))
    assert _call_static(lib, V, M, tau, q, A_log, B, C, D, dt, y, h, FTILE=FTILE) == 0, lib.tssm_last_error()
    torch.cuda.synchronize()
    assert rel_err(y, y_ref) < TOL_FP32
    assert rel_err(h, h_ref) < TOL_FP32


# (N, FTILE): the chunked scan with its blocked table (N <= 16, 32-feature runs
# inside tiles), and the two cases that take the raw-table kernel instead
# (N > 16; a tile width that is not a multiple of 32).
@pytest.mark.parametrize("N,FTILE", [(16, 128), (32, 128), (16, 48)])
def test_static_scratch_matches_workspace_entry_point(cuda_ops, N, FTILE):
    from triton_ssm_b200 import _lib
    lib = _lib.load_library()
    inputs = _inputs(N=N)
    for _ in range(2):   # two calls in a row share (and reuse) the static scratch
        _check_against_workspace_entry(cuda_ops, lib, inputs, FTILE)


def test_static_scratch_larger_then_smaller_problem(cuda_ops):
    """A smaller problem after a larger one reads none of the larger one's
    leftovers in the shared array."""
    from triton_ssm_b200 import _lib
    lib = _lib.load_library()
    _check_against_workspace_entry(cuda_ops, lib, _inputs(seed=5, Bt=4, T=300, Lq=500), 128)
    _check_against_workspace_entry(cuda_ops, lib, _inputs(seed=6, Bt=2, T=100, Lq=150), 128)
    _check_against_workspace_entry(cuda_ops, lib, _inputs(seed=7, Bt=1, T=40, Dm=32, Lq=33), 32)


def test_static_scratch_through_the_python_operator(cuda_ops):
    V, M, tau, q, A_log, B, C, D, dt = _inputs(seed=9)
    y_ref = cuda_ops.fused_interp_ssm(V, M, tau, A_log, B, C, q=q, dt=dt, D=D)
    y = cuda_ops.fused_interp_ssm(V, M, tau, A_log, B, C, q=q, dt=dt, D=D, static_scratch=True)
    assert rel_err(y, y_ref) < TOL_FP32
    with pytest.raises(ValueError):   # the wrapper's shape checks apply on this path too
        cuda_ops.fused_interp_ssm(V, M[:, :-1], tau, A_log, B, C, q=q, dt=dt, static_scratch=True)


def test_static_scratch_rejects_oversized_problem(cuda_ops):
    from triton_ssm_b200 import _lib
    lib = _lib.load_library()
    V, M, tau, q, A_log, B, C, D, dt = _inputs(Bt=1, T=8, Dm=8, N=4, Lq=8)
    # 64 rows x 2048 queries x 4 tiles of table entries is far beyond 8 MiB
    need = lib.tssm_interp_ssm_workspace_size(64, 2048, 512, 65536, 128)
    assert need > (8 << 20)
    P = ctypes.c_void_p
    st = lib.tssm_interp_ssm_static_scratch(
        P(V.data_ptr()), P(M.data_ptr()), P(tau.data_ptr()), P(q.data_ptr()), P(A_log.data_ptr()),
        P(B.data_ptr()), P(C.data_ptr()), P(D.data_ptr()), P(dt.data_ptr()), P(V.data_ptr()), P(0), P(0),
        64, 2048, 512, 4, 65536, 10, 128, 3, P(torch.cuda.current_stream().cuda_stream))
    assert st == 1
    assert b"static scratch" in lib.tssm_last_error()
