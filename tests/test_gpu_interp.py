"""GPU parity of the interpolation kernels: reference-exact standalone
interpolation and single step (golden fixtures from the reference kernels),
and the fused interpolation + N-state scan against the CPU oracle."""
import pytest
import torch

import oracle
from conftest import TOL_FP32, load_golden, parity, rel_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def cu(t):
    return t.to(dev)


@pytest.mark.parametrize("dtn,dty", [("fp32", torch.float32), ("bf16", torch.bfloat16), ("fp16", torch.float16)])
def test_interp_golden(cuda_ops, dtn, dty):
    g = load_golden("interp_" + dtn)
    vh = cuda_ops.fused_time_aware_interp(cu(g["V"].to(dty)), cu(g["M"]), cu(g["tau"]))
    if dty == torch.float32:
        assert torch.equal(vh.cpu(), g["Vhat"])        # bit-exact with the reference's fp32 arithmetic
    else:
        assert rel_err(vh, g["Vhat"]) < 1e-2


def test_interp_float_mask_and_strides(cuda_ops):
    g = load_golden("interp_fp32")
    V = cu(g["V"])
    big = torch.zeros(V.shape[0], V.shape[1] * 2, V.shape[2], device=dev)
    big[:, ::2] = V
    vh = cuda_ops.fused_time_aware_interp(big[:, ::2], cu(g["M"].float()), cu(g["tau"]))
    assert torch.equal(vh.cpu(), g["Vhat"])


@pytest.mark.parametrize("F,K,FTILE", [(200, 10, 128), (7, 3, 4), (300, 1, 64)])
def test_interp_random_vs_oracle(cuda_ops, F, K, FTILE):
    gen = torch.Generator().manual_seed(F + K)
    Bt, T = 3, 150
    V = torch.randn(Bt, T, F, generator=gen)
    M = (torch.rand(Bt, T, F, generator=gen) < 0.1).to(torch.uint8)
    tau = torch.cumsum(torch.rand(Bt, T, generator=gen), 1)
    vh = cuda_ops.fused_time_aware_interp(cu(V), cu(M), cu(tau), K=K, FTILE=FTILE)
    ref = oracle.time_aware_interp(V, M, tau, K=K, FTILE=FTILE)
    assert torch.equal(vh.cpu(), ref)


def test_interp_step_golden(cuda_ops):
    g = load_golden("interp_step_seq")
    V, M, tau = cu(g["V"]), cu(g["M"]), cu(g["tau"])
    h = cu(g["h0"])
    Vhat = torch.zeros_like(V)
    for t in range(V.shape[1]):
        h = cuda_ops.fused_interp_ssm_step(V, M, tau, cu(g["Abar"]), cu(g["Bbar"]), h, Vhat=Vhat, t_cur=t)
        assert torch.equal(h.cpu(), g["h_seq"][t]), t
    assert torch.equal(Vhat.cpu(), g["Vhat"])


def test_interp_ssm_obsgrid_golden(cuda_ops):
    g = load_golden("interp_ssm_obsgrid")
    y, h, vh = cuda_ops.fused_interp_ssm(cu(g["V"]), cu(g["M"]), cu(g["tau"]), cu(g["A_log"]), cu(g["B"]),
                                         cu(g["C"]), dt=cu(g["dt"]), return_state=True, return_vhat=True)
    assert torch.equal(vh.cpu(), g["Vhat"])
    assert rel_err(y, g["y"]) < TOL_FP32
    assert rel_err(h, g["h_last"]) < TOL_FP32


def make_c3(Bt, T, Dm, N, Lq, seed, p_obs=0.7):
    gen = torch.Generator().manual_seed(seed)
    V = torch.randn(Bt, T, Dm, generator=gen)
    M = (torch.rand(Bt, T, Dm, generator=gen) < p_obs).to(torch.uint8)
    tau = torch.cumsum(torch.empty(Bt, T).exponential_(1.0, generator=gen), 1)
    A_log = torch.log(torch.arange(1, N + 1, dtype=torch.float32)).repeat(Dm, 1)
    B = torch.randn(Dm, N, generator=gen) / N ** 0.5
    C = torch.randn(Dm, N, generator=gen) / N ** 0.5
    D = torch.randn(Dm, generator=gen)
    return V, M, tau, A_log, B, C, D


@pytest.mark.parametrize("Bt,T,Dm,N,Lq,p_obs", [(2, 300, 256, 16, 600, 0.7), (3, 100, 70, 5, 257, 0.02),
                                                 (1, 64, 33, 64, 64, 0.3), (4, 300, 64, 16, 500, 0.7),
                                                 (2, 90, 192, 16, 120, 0.02),
                                                 # sparse queries: every 32-query block spans more rows than
                                                 # are staged, so values are gathered from global memory
                                                 (2, 2000, 64, 16, 100, 0.7),
                                                 (2, 300, 96, 5, 700, 0.3), (1, 200, 64, 3, 333, 0.7),
                                                 (3, 150, 32, 16, 33, 0.7), (1, 40, 32, 16, 5, 0.7)])
def test_interp_ssm_query_grid_vs_oracle(cuda_ops, Bt, T, Dm, N, Lq, p_obs):
    V, M, tau, A_log, B, C, D = make_c3(Bt, T, Dm, N, Lq, seed=T + N, p_obs=p_obs)
    # the same query times on both sides (a device-built grid may differ in the last ulp)
    q = oracle.linspace_queries(tau, Lq)
    dt = (tau[:, -1] - tau[:, 0]) / (Lq - 1)
    # a workspace holding garbage: every flag and table entry must be written before it is read
    need = cuda_ops.interp_ssm_workspace_bytes(Bt, T, Dm, Lq)
    ws = torch.full((need,), 0xA5, dtype=torch.uint8, device=dev)
    y, h, vh = cuda_ops.fused_interp_ssm(cu(V), cu(M), cu(tau), cu(A_log), cu(B), cu(C), q=cu(q), dt=cu(dt),
                                         D=cu(D), return_state=True, return_vhat=True, workspace=ws)
    ry, rh, rvh = oracle.interp_ssm(V, M, tau, A_log, B, C, dt, q=q, D=D, return_vhat=True)
    assert torch.equal(vh.cpu(), rvh)
    assert rel_err(y, ry) < TOL_FP32
    assert rel_err(h, rh) < TOL_FP32


@pytest.mark.parametrize("FTILE,p_obs", [(32, 0.05), (64, 0.02), (96, 0.7), (48, 0.3)])
def test_interp_ssm_feature_tiles(cuda_ops, FTILE, p_obs):
    """Neighbour tables per tile of FTILE features: each run of 32 features reads
    its own tile's table (FTILE 96 puts runs of one CTA in different tiles)."""
    Bt, T, Dm, N, Lq = 2, 400, 192, 16, 900
    V, M, tau, A_log, B, C, D = make_c3(Bt, T, Dm, N, Lq, seed=FTILE, p_obs=p_obs)
    q = oracle.linspace_queries(tau, Lq)
    dt = (tau[:, -1] - tau[:, 0]) / (Lq - 1)
    y, h, vh = cuda_ops.fused_interp_ssm(cu(V), cu(M), cu(tau), cu(A_log), cu(B), cu(C), q=cu(q), dt=cu(dt),
                                         D=cu(D), FTILE=FTILE, return_state=True, return_vhat=True)
    ry, rh, rvh = oracle.interp_ssm(V, M, tau, A_log, B, C, dt, q=q, D=D, FTILE=FTILE, return_vhat=True)
    assert torch.equal(vh.cpu(), rvh)
    assert rel_err(y, ry) < TOL_FP32
    assert rel_err(h, rh) < TOL_FP32


@pytest.mark.parametrize("dt_scale", [1e-3, 1.0])
def test_interp_ssm_slow_and_fast_decay(cuda_ops, dt_scale):
    """A small dt (Abar near 1, slow decay) makes the scan carry state across the
    whole query range; a large one forgets within a few queries."""
    Bt, T, Dm, N, Lq = 2, 500, 64, 16, 2000
    V, M, tau, A_log, B, C, D = make_c3(Bt, T, Dm, N, Lq, seed=11)
    q = oracle.linspace_queries(tau, Lq)
    dt = torch.full((Bt,), dt_scale)
    y, h = cuda_ops.fused_interp_ssm(cu(V), cu(M), cu(tau), cu(A_log), cu(B), cu(C), q=cu(q), dt=cu(dt),
                                     D=cu(D), return_state=True)
    ry, rh = oracle.interp_ssm(V, M, tau, A_log, B, C, dt, q=q, D=D)
    assert rel_err(y, ry) < TOL_FP32
    assert rel_err(h, rh) < TOL_FP32


def test_interp_ssm_regular_grid_argument(cuda_ops):
    V, M, tau, A_log, B, C, D = make_c3(2, 200, 64, 16, 400, seed=8)
    y = cuda_ops.fused_interp_ssm(cu(V), cu(M), cu(tau), cu(A_log), cu(B), cu(C), L_q=400)
    q = oracle.linspace_queries(tau, 400)
    dt = (tau[:, -1] - tau[:, 0]) / 399
    ry, _ = oracle.interp_ssm(V, M, tau, A_log, B, C, dt, q=q)
    assert rel_err(y, ry) < TOL_FP32


def test_interp_ssm_config3_full_size(cuda_ops):
    """Config 3 at full size (B32 L_obs 2048 -> L_q 4096, D256 N16) against the oracle
    on a subset of rows (the oracle is a sequential CPU loop)."""
    V, M, tau, A_log, B, C, D = make_c3(32, 2048, 256, 16, 4096, seed=3)
    q = oracle.linspace_queries(tau, 4096)
    dt = (tau[:, -1] - tau[:, 0]) / 4095
    y, h = cuda_ops.fused_interp_ssm(cu(V), cu(M), cu(tau), cu(A_log), cu(B), cu(C), q=cu(q), dt=cu(dt),
                                     return_state=True)
    rows = [0, 17, 31]
    ry, rh = oracle.interp_ssm(V[rows], M[rows], tau[rows], A_log, B, C, dt[rows], q=q[rows])
    parity("config 3 y  (B32 Lobs2048->Lq4096 D256 N16, f32; rows 0,17,31)", y[rows], ry, TOL_FP32)
    parity("config 3 h_last", h[rows], rh, TOL_FP32)


def test_interp_ssm_rejects_bad_args(cuda_ops):
    V, M, tau, A_log, B, C, D = make_c3(1, 10, 8, 4, 10, seed=0)
    with pytest.raises(ValueError):
        cuda_ops.fused_interp_ssm(cu(V), cu(M), cu(tau), cu(A_log), cu(B), cu(C))   # index mode, no dt
