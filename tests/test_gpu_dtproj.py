"""GPU parity of the delta-t projection (discretize_kernel.py:165-213) and of
its fusion into the per-channel ZOH discretisation, against the CPU oracle on
the same seeded inputs.  The reference kernel does not compile, so the oracle's
restatement is the only pin for this function."""
import pytest
import torch

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def cu(t):
    return t.to(dev)


def _inputs(Bt, T, H, R, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    dt_raw = torch.randn(Bt, T, R, generator=g) * scale
    W = torch.randn(R, H, generator=g) / R ** 0.5
    bias = torch.randn(H, generator=g) - 3.0
    A_log = torch.log(torch.empty(H).uniform_(0.5, 16, generator=g))
    B = torch.randn(Bt, T, H, generator=g)
    return dt_raw, W, bias, A_log, B


@pytest.mark.parametrize("Bt,T,H,R", [(1, 1, 1, 1), (2, 33, 37, 5), (3, 64, 1024, 64), (2, 50, 130, 256),
                                      (1, 7, 4096, 16)])
def test_dt_project_vs_oracle(cuda_ops, Bt, T, H, R):
    dt_raw, W, bias, _, _ = _inputs(Bt, T, H, R, seed=H + R)
    for lo, hi in ((1e-3, 1e-1), (1e-4, 10.0)):
        dt = cuda_ops.dt_project_softplus(cu(dt_raw), cu(W), cu(bias), lo, hi)
        ref = oracle.dt_project_softplus(dt_raw, W, bias, lo, hi)
        assert rel_err(dt, ref) < 1e-5
        lo32, hi32 = (float(torch.tensor(v, dtype=torch.float32)) for v in (lo, hi))
        assert float(dt.min()) >= lo32 and float(dt.max()) <= hi32


def test_dt_project_overflow_clamps(cuda_ops):
    """A large pre-activation overflows exp to inf, as in the reference, and clamps to DT_MAX."""
    dt_raw, W, bias, _, _ = _inputs(2, 9, 40, 8, seed=1, scale=200.0)
    dt = cuda_ops.dt_project_softplus(cu(dt_raw), cu(W), cu(bias), 1e-3, 0.5)
    ref = oracle.dt_project_softplus(dt_raw, W, bias, 1e-3, 0.5)
    assert torch.isfinite(dt).all()
    assert rel_err(dt, ref) < 1e-5


@pytest.mark.parametrize("Bt,T,H,R", [(2, 17, 37, 5), (3, 64, 1024, 64), (1, 40, 131, 32)])
def test_discretize_dtproj_vs_composition(cuda_ops, Bt, T, H, R):
    dt_raw, W, bias, A_log, B = _inputs(Bt, T, H, R, seed=T + R)
    Ab, Bb, dt = cuda_ops.zoh_discretize_dtproj(cu(A_log), cu(B), cu(dt_raw), cu(W), cu(bias), 1e-4, 2.0,
                                                return_dt=True)
    ref_dt = oracle.dt_project_softplus(dt_raw, W, bias, 1e-4, 2.0)
    rA, rB = oracle.zoh_discretize_dt(A_log, B, ref_dt)
    assert rel_err(dt, ref_dt) < 1e-5
    assert rel_err(Ab, rA) < 1e-5
    assert rel_err(Bb, rB) < 1e-5
    # without the dt output the fused form may take the tensor-core kernel (another summation order)
    Ab2, Bb2 = cuda_ops.zoh_discretize_dtproj(cu(A_log), cu(B), cu(dt_raw), cu(W), cu(bias), 1e-4, 2.0)
    assert rel_err(Ab2, rA) < 1e-5 and rel_err(Bb2, rB) < 1e-5
    assert rel_err(Ab2, Ab) < 1e-5 and rel_err(Bb2, Bb) < 1e-5


@pytest.mark.parametrize("Bt,T,H,R", [(16, 64, 1024, 64), (3, 100, 200, 64), (2, 130, 68, 32), (1, 300, 520, 12),
                                      (2, 40, 37, 8), (4, 96, 100, 16)])
def test_dtproj_tensor_core_shapes(cuda_ops, Bt, T, H, R):
    """Shapes the tcgen05 kernel takes (R <= 64, R a multiple of 4), against the
    oracle: partial 128-row and 128-channel tiles, K padded past R, warp blocks
    split between the 16-byte staged epilogue and the checked one, and H % 4 != 0
    (every block on the checked epilogue)."""
    dt_raw, W, bias, A_log, B = _inputs(Bt, T, H, R, seed=Bt * T + H + R)
    ref_dt = oracle.dt_project_softplus(dt_raw, W, bias, 1e-3, 0.1)
    rA, rB = oracle.zoh_discretize_dt(A_log, B, ref_dt)
    Ab, Bb = cuda_ops.zoh_discretize_dtproj(cu(A_log), cu(B), cu(dt_raw), cu(W), cu(bias), 1e-3, 0.1)
    assert rel_err(Ab, rA) < 1e-5 and rel_err(Bb, rB) < 1e-5
    dt = cuda_ops.dt_project_softplus(cu(dt_raw), cu(W), cu(bias), 1e-3, 0.1)
    assert rel_err(dt, ref_dt) < 1e-5


def test_dt_project_rejects_bad_args(cuda_ops):
    z = lambda *s: torch.zeros(*s, device=dev)
    with pytest.raises(ValueError):
        cuda_ops.dt_project_softplus(z(2, 3, 4), z(5, 6), z(6))
    with pytest.raises(ValueError):
        cuda_ops.dt_project_softplus(z(2, 3, 300), z(300, 6), z(6))   # R > 256, refused by the library
    with pytest.raises(ValueError):
        cuda_ops.dt_project_softplus(z(2, 3, 4), z(4, 6), z(6), 1.0, 0.5)


@pytest.mark.parametrize("Bt,T,H,R", [(1, 1, 4, 4), (1, 5, 20, 60), (3, 77, 300, 40), (2, 64, 256, 64)])
def test_dtproj_tensor_core_small_and_odd(cuda_ops, Bt, T, H, R):
    """Tiny and odd shapes on the tcgen05 kernel: one row, fewer than 32 rows or
    channels, K padded past R inside a 32-wide atom, whole and partial blocks;
    both outputs of the fused form and the dt-only form, with and without dt."""
    dt_raw, W, bias, A_log, B = _inputs(Bt, T, H, R, seed=7 * T + H + R)
    ref_dt = oracle.dt_project_softplus(dt_raw, W, bias, 1e-3, 0.1)
    rA, rB = oracle.zoh_discretize_dt(A_log, B, ref_dt)
    Ab, Bb, dt = cuda_ops.zoh_discretize_dtproj(cu(A_log), cu(B), cu(dt_raw), cu(W), cu(bias), 1e-3, 0.1,
                                                return_dt=True)
    assert rel_err(Ab, rA) < 1e-5 and rel_err(Bb, rB) < 1e-5 and rel_err(dt, ref_dt) < 1e-5
    dt2 = cuda_ops.dt_project_softplus(cu(dt_raw), cu(W), cu(bias), 1e-3, 0.1)
    assert rel_err(dt2, ref_dt) < 1e-5


def test_dtproj_tensor_core_matches_cuda_core_kernel(cuda_ops):
    """dt_rank 64 takes the tcgen05 kernel; the same problem padded to dt_rank 65
    with a zero column and a zero row of W takes the CUDA-core kernel.  The two
    agree to f32 accuracy (different summation order, different exp/log forms)."""
    Bt, T, H, R = 4, 130, 520, 64
    dt_raw, W, bias, A_log, B = _inputs(Bt, T, H, R, seed=11)
    dt_raw65 = torch.cat([dt_raw, torch.zeros(Bt, T, 1)], dim=2)
    W65 = torch.cat([W, torch.zeros(1, H)], dim=0)
    a_tc, b_tc = cuda_ops.zoh_discretize_dtproj(cu(A_log), cu(B), cu(dt_raw), cu(W), cu(bias), 1e-3, 0.1)
    a_cc, b_cc = cuda_ops.zoh_discretize_dtproj(cu(A_log), cu(B), cu(dt_raw65), cu(W65), cu(bias), 1e-3, 0.1)
    assert rel_err(a_tc, a_cc) < 1e-5 and rel_err(b_tc, b_cc) < 1e-5
    d_tc = cuda_ops.dt_project_softplus(cu(dt_raw), cu(W), cu(bias), 1e-3, 0.1)
    d_cc = cuda_ops.dt_project_softplus(cu(dt_raw65), cu(W65), cu(bias), 1e-3, 0.1)
    assert rel_err(d_tc, d_cc) < 1e-5


def test_dtproj_wide_rows_fall_back_to_cuda_cores(cuda_ops):
    """A single 128-row block across more channel blocks than SMs would give a
    CTA three channel blocks: the tensor-core launcher declines it and the
    CUDA-core kernel computes it, with the same result as the oracle."""
    Bt, T, H, R = 1, 128, 19000, 64
    dt_raw, W, bias, A_log, B = _inputs(Bt, T, H, R, seed=19)
    ref_dt = oracle.dt_project_softplus(dt_raw, W, bias, 1e-3, 0.1)
    rA, rB = oracle.zoh_discretize_dt(A_log, B, ref_dt)
    Ab, Bb = cuda_ops.zoh_discretize_dtproj(cu(A_log), cu(B), cu(dt_raw), cu(W), cu(bias), 1e-3, 0.1)
    assert rel_err(Ab, rA) < 1e-5 and rel_err(Bb, rB) < 1e-5
