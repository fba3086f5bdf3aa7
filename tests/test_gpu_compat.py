"""The reference's own launch syntax, kernel[grid](...), with its argument
lists, through triton_ssm_b200.compat — on the golden fixtures."""
import pytest
import torch

from conftest import load_golden, rel_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def test_compat_discretize(cuda_ops):
    from triton_ssm_b200.compat import discretize_kernel as dk
    g = load_golden("discretize_fp32")
    A, Bc, dt = (g[k].to(dev) for k in ("A_log", "B", "dt"))
    Bsz, T, H = Bc.shape
    Ab, Bb = torch.empty_like(Bc), torch.empty_like(Bc)
    dk.zoh_discretize_diag_kernel[(Bsz, T, 2)](A, Bc, dt, Ab, Bb, Bsz, T, H, *Bc.stride(), *dt.stride(),
                                               *Ab.stride(), *Bb.stride(), BLOCK_H=32)
    assert rel_err(Ab, g["Abar"]) < 1e-5 and rel_err(Bb, g["Bbar"]) < 1e-5


def test_compat_interp_and_step(cuda_ops):
    from triton_ssm_b200.compat import fused_interp_kernel as fik, fused_ssm_interp as fsi
    g = load_golden("interp_fp32")
    V, M, tau = (g[k].to(dev) for k in ("V", "M", "tau"))
    Bsz, T, F = V.shape
    Vh = torch.empty_like(V)
    fik.fused_time_aware_interp_kernel[(Bsz, T, 2)](V, M, tau, Vh, Bsz, T, F, *V.stride(), *M.stride(), *tau.stride(),
                                                    *Vh.stride(), K=10, FTILE=128)
    assert torch.equal(Vh.cpu(), g["Vhat"])
    g = load_golden("interp_step_seq")
    V, M, tau, Ab, Bb = (g[k].to(dev) for k in ("V", "M", "tau", "Abar", "Bbar"))
    Bsz, T, F = V.shape
    h = g["h0"].to(dev)
    Vhat = torch.zeros_like(V)
    for t in range(T):
        h_out = torch.empty_like(h)
        fsi.fused_interp_ssm_step_kernel[(Bsz, 2)](V, M, tau, Ab, Bb, h, Vhat, h_out, Bsz, T, F, *V.stride(),
                                                  *M.stride(), *tau.stride(), *Vhat.stride(), *h.stride(),
                                                  *h_out.stride(), t, K=10, FTILE=128)
        h = h_out
    assert torch.equal(h.cpu(), g["h_seq"][-1])


def test_compat_streaming_and_scan(cuda_ops):
    from triton_ssm_b200.compat import streaming_inference_kernel as sik, ssm_scan
    g = load_golden("stream_inplace_fp32")
    vh, h, Ab, Bb, C, D = (g[k].to(dev) for k in ("vhat", "h_in", "Abar", "Bbar", "C", "D"))
    y = torch.empty_like(vh)
    Bsz, H = vh.shape
    sik.streaming_ssm_inplace_kernel[(Bsz, 2)](vh, h, Ab, Bb, C, D, y, Bsz, H, *vh.stride(), *h.stride(),
                                               *C.stride(), BLOCK_H=64)
    assert rel_err(h, g["h_out"]) < 1e-6 and rel_err(y, g["y"]) < 1e-6
    g = load_golden("ssm_forward_a")
    yy, hh = ssm_scan.ssm_forward(*(g[k].to(dev) for k in ("u", "A", "B", "C", "D")), BLK=64)
    assert rel_err(yy, g["y"]) < 1e-4


def _pow2(n):
    p = 1
    while p < n:
        p *= 2
    return p


def test_compat_ssm_forward_four_launches(cuda_ops):
    """ssm_forward's own four launches (ssm_scan.py:239-264) through the shims,
    on the golden minted from the reference."""
    from triton_ssm_b200.compat import ssm_scan as ss
    g = load_golden("ssm_forward_a")
    u, A, B, C, D = (g[k].to(dev) for k in ("u", "A", "B", "C", "D"))
    Bsz, L, H = u.shape
    BLK = 64
    nblk = _pow2((L + BLK - 1) // BLK)
    loc_a, loc_x, h, y = (torch.empty_like(A) for _ in range(4))
    carry = torch.empty(2 * Bsz * H * nblk, device=dev)
    ss.ssm_fwd_local_kernel[(Bsz * H, nblk)](u, A, B, loc_a, loc_x, carry, Bsz, L, H, BLK, nblk)
    ss.ssm_carry_scan_kernel[(Bsz * H,)](carry, Bsz * H, nblk)
    ss.ssm_fwd_apply_kernel[(Bsz * H, nblk)](loc_a, loc_x, carry, h, Bsz, L, H, BLK, nblk)
    ss.ssm_output_kernel[(Bsz * H, nblk)](h, C, D, u, y, Bsz, L, H, BLK)
    assert rel_err(h, g["h"]) < 1e-4 and rel_err(y, g["y"]) < 1e-4


def test_compat_ssm_backward_three_launches(cuda_ops):
    """ssm_backward's launches (ssm_scan.py:267-289) through the shims, on the
    golden minted from the reference, and the host function itself."""
    from triton_ssm_b200.compat import ssm_scan as ss
    g = load_golden("ssm_backward")
    u, A, B, C, h, dY = (g[k].to(dev) for k in ("u", "A", "B", "C", "h", "dY"))
    Bsz, L, H = u.shape
    BLK = 32
    nblk = _pow2((L + BLK - 1) // BLK)
    loc_a, loc_dh, du, dA, dB, dC = (torch.empty_like(A) for _ in range(6))
    carry = torch.empty(2 * Bsz * H * nblk, device=dev)
    ss.ssm_bwd_local_kernel[(Bsz * H, nblk)](A, C, dY, loc_a, loc_dh, carry, Bsz, L, H, BLK, nblk)
    ss.ssm_bwd_carry_scan_kernel[(Bsz * H,)](carry, Bsz * H, nblk)
    ss.ssm_bwd_apply_kernel[(Bsz * H, nblk)](loc_a, loc_dh, carry, u, A, B, h, dY, du, dA, dB, dC, Bsz, L, H, BLK,
                                             nblk)
    for name, t in (("du", du), ("dA", dA), ("dB", dB), ("dC", dC)):
        assert rel_err(t, g[name]) < 1e-4, name
    du2, dA2, dB2, dC2 = ss.ssm_backward(u, A, B, C, h, dY)
    assert rel_err(du2, g["du"]) < 1e-4 and rel_err(dA2, g["dA"]) < 1e-4


@pytest.mark.parametrize("dty", [torch.float32, torch.bfloat16])
def test_compat_multihead_three_launches(cuda_ops, dty):
    """multihead_ssm_kernel.py's three launches compose to the diagonal
    multi-head scan: against the golden (composed from the reference's own
    kernels) and against multihead_ssm(mode="diag")."""
    from triton_ssm_b200.compat import multihead_ssm_kernel as mk
    g = load_golden("mh_diag_composed")
    u = g["x"].to(dev).to(dty)
    A_log, dt, D = (g[k].to(dev) for k in ("A_log", "dt", "D"))
    Bm, Cm = g["B"].to(dev).to(dty), g["C"].to(dev).to(dty)
    Bsz, L, H = u.shape
    nh, hd = A_log.shape
    BLK = 16
    nblk = _pow2((L + BLK - 1) // BLK)
    rows = Bsz * nh * hd
    loc_a = torch.empty(Bsz, L, nh, hd, device=dev)
    loc_x = torch.empty_like(loc_a)
    carry = torch.empty(2 * rows * nblk, device=dev)
    y = torch.empty_like(u)
    mk.multihead_ssm_fwd_local_kernel[(Bsz * nh, nblk)](
        u, A_log, Bm, Cm, dt, loc_a, loc_x, carry, Bsz, L, H, nh, hd, *u.stride(), *A_log.stride(), *Bm.stride(),
        *Cm.stride(), *dt.stride(), BLK_L=BLK, NBLK=nblk, HEAD_DIM=hd)
    mk.multihead_ssm_carry_scan_kernel[(rows,)](carry, rows, nblk)
    mk.multihead_ssm_output_kernel[(Bsz * nh, nblk)](
        loc_a, loc_x, carry, Cm, D, u, y, Bsz, L, H, nh, hd, *u.stride(), *Cm.stride(), BLK_L=BLK, NBLK=nblk,
        HEAD_DIM=hd)
    tol = 1e-4 if dty == torch.float32 else 2e-2
    fused = cuda_ops.multihead_ssm(u, A_log, Bm, Cm, dt, D, mode="diag")
    assert rel_err(y, fused) < tol
    if dty == torch.float32:
        assert rel_err(y, g["y"]) < tol


def test_compat_discretize_bwd_and_dtproj(cuda_ops):
    import oracle
    from triton_ssm_b200.compat import discretize_kernel as dk
    g = load_golden("discretize_bwd")
    A, Bc, dt, Ab, dAb, dBb = (g[k].to(dev) for k in ("A_log", "B", "dt", "Abar", "dAbar", "dBbar"))
    Bsz, T, H = Bc.shape
    dA = torch.zeros(H, device=dev)
    dB, ddt = torch.empty_like(Bc), torch.empty_like(dt)
    dk.zoh_discretize_bwd_kernel[(Bsz, T, 1)](A, Bc, dt, Ab, dAb, dBb, dA, dB, ddt, Bsz, T, H, *Bc.stride(),
                                              *dt.stride(), *Ab.stride(), *dBb.stride(), BLOCK_H=32)
    assert rel_err(dA, g["dA_log"]) < 1e-4 and rel_err(dB, g["dB"]) < 1e-5 and rel_err(ddt, g["ddt"]) < 1e-4
    gen = torch.Generator().manual_seed(3)
    dt_raw = torch.randn(2, 7, 16, generator=gen)
    W = torch.randn(16, 40, generator=gen) / 4
    bias = torch.randn(40, generator=gen)
    out = torch.empty(2, 7, 40, device=dev)
    dk.dt_project_softplus_kernel[(2, 7, 1)](dt_raw.to(dev), W.to(dev), bias.to(dev), out, 2, 7, 40, 16,
                                             *dt_raw.stride(), *W.stride(), *out.stride(), DT_MIN=1e-3, DT_MAX=0.1,
                                             BLOCK_H=64, BLOCK_R=16)
    ref = oracle.dt_project_softplus(dt_raw, W, bias, 1e-3, 0.1)
    assert rel_err(out, ref) < 1e-5


def test_compat_ring_and_pool(cuda_ops):
    import oracle
    from triton_ssm_b200.compat import streaming_inference_kernel as sik
    g = load_golden("ring_stream")
    rV, rM, rT, rH, h = (g[k].clone().to(dev) for k in ("ring_V", "ring_M", "ring_tau", "ring_head", "h0"))
    K = int(g["K"])
    Bsz, H = h.shape
    for e in range(g["v"].shape[0]):
        v, m, tau, C = (g[k][e].to(dev) for k in ("v", "m", "tau", "C"))
        y = torch.empty_like(v)
        sik.streaming_interp_then_ssm_kernel[(Bsz, 1)](
            rV, rM, rT, rH, v, m, tau, h, g["Abar"].to(dev), g["Bbar"].to(dev), C, g["D"].to(dev), y, Bsz, H, K,
            *rV.stride(), *v.stride(), *h.stride(), *C.stride(), BLOCK_H=32, KRING=K + 1)
        assert rel_err(y, g["y"][e]) < 1e-6 and rel_err(h, g["h"][e]) < 1e-6
    assert torch.equal(rV.cpu(), g["ring_V_final"]) and torch.equal(rH.cpu(), g["ring_head_final"])
    gen = torch.Generator().manual_seed(4)
    x = torch.randn(3, 50, 24, generator=gen)
    W = torch.randn(24, generator=gen)
    bias = torch.tensor(0.25)
    out = torch.empty(3, device=dev)
    sik.mean_pool_logit_kernel[(3,)](x.to(dev), W.to(dev), bias.to(dev), out, 3, 50, 24, *x.stride(), BLOCK_H=32,
                                     BLOCK_T=16)
    assert rel_err(out, oracle.mean_pool_logit(x, W, bias)) < 1e-5
