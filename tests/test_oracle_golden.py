"""The CPU oracle against the golden fixtures minted from the reference's own
kernels (tests/golden/make_golden.py).  CPU only."""
import torch

import oracle
from conftest import TOL_BF16, TOL_FP32, load_golden, rel_err


def test_discretize_fp32():
    g = load_golden("discretize_fp32")
    Ab, Bb = oracle.zoh_discretize(g["A_log"], g["B"], g["dt"])
    assert rel_err(Ab, g["Abar"]) < 1e-6
    assert rel_err(Bb, g["Bbar"]) < 1e-6
    # elementwise: exp(x)-1 cancels in fp32 just above the 1e-5 branch point, so
    # two exp implementations may differ there by a few ulp of 1.0 (scaled by
    # |B/a|); everywhere else they agree to fp32 rounding.
    a = -torch.exp(g["A_log"])
    bound = 4 * 2.0 ** -23 * (g["B"].abs() / a.abs()) + 1e-6 * g["Bbar"].abs()
    assert ((Bb - g["Bbar"]).abs() <= bound).all()


def test_discretize_bf16():
    g = load_golden("discretize_bf16")
    Ab, Bb = oracle.zoh_discretize(g["A_log"], g["B"].bfloat16(), g["dt"], variant="bf16")
    assert rel_err(Ab, g["Abar"]) < 1e-2
    assert rel_err(Bb, g["Bbar"]) < 1e-2
    # bf16 rounding of the same fp32 value: at most one bf16 ulp apart
    assert (Ab.float() - g["Abar"]).abs().max() <= 2 ** -8


def test_ssm_forward():
    for name in ("ssm_forward_a", "ssm_forward_b"):
        g = load_golden(name)
        y, h = oracle.ssm_forward(g["u"], g["A"], g["B"], g["C"], g["D"])
        assert rel_err(y, g["y"]) < TOL_FP32, name
        assert rel_err(h, g["h"]) < TOL_FP32, name


def test_c1_pair_selective_scan():
    g = load_golden("c1_pair")
    y, h = oracle.selective_scan(g["x"], g["dt"], g["A_log"], g["B"], g["C"], g["D"])
    assert rel_err(y, g["y"]) < TOL_FP32
    assert rel_err(h, g["h_last"]) < TOL_FP32


def test_ssd_composed():
    g = load_golden("ssd_composed")
    y, h = oracle.ssd_scan(g["x"], g["dt"], g["A_log"], g["B"], g["C"], g["D"])
    assert rel_err(y, g["y"]) < TOL_FP32
    assert rel_err(h, g["h_last"]) < TOL_FP32
    for Q in (7, 16, 64):
        yc, hc = oracle.ssd_scan_chunked(g["x"], g["dt"], g["A_log"], g["B"], g["C"], g["D"], chunk=Q)
        assert rel_err(yc, g["y"]) < TOL_FP32
        assert rel_err(hc, g["h_last"]) < TOL_FP32


def test_ssd_sharded_composition():
    g = load_golden("ssd_composed")
    x, dt, A_log, B, C, D = (g[k] for k in ("x", "dt", "A_log", "B", "C", "D"))
    L = x.shape[1]
    cuts = [0, 13, 27, L]
    parts = [oracle.ssd_scan(x[:, a:b], dt[:, a:b], A_log, B[:, a:b], C[:, a:b], D)
             for a, b in zip(cuts[:-1], cuts[1:])]
    carries = oracle.ssd_sharded_compose(parts, A_log, [dt[:, a:b] for a, b in zip(cuts[:-1], cuts[1:])])
    ys = []
    for (a, b), carry in zip(zip(cuts[:-1], cuts[1:]), carries):
        yy, _ = oracle.ssd_scan(x[:, a:b], dt[:, a:b], A_log, B[:, a:b], C[:, a:b], D, h0=carry)
        ys.append(yy)
    assert rel_err(torch.cat(ys, 1), g["y"]) < TOL_FP32


def test_multihead_diag():
    g = load_golden("mh_diag_composed")
    y, _ = oracle.multihead_diag(g["x"], g["A_log"], g["B"], g["C"], g["dt"], g["D"])
    assert rel_err(y, g["y"]) < TOL_FP32


def test_interp_three_dtypes():
    for dtn, dty, tol in (("fp32", torch.float32, 1e-6), ("bf16", torch.bfloat16, 1e-2),
                          ("fp16", torch.float16, 2e-3)):
        g = load_golden("interp_" + dtn)
        vh = oracle.time_aware_interp(g["V"].to(dty), g["M"], g["tau"])
        assert rel_err(vh, g["Vhat"]) < tol, dtn


def test_interp_query_mode_equals_index_mode_on_obs_times():
    g = load_golden("interp_fp32")
    V, M, tau = g["V"], g["M"], g["tau"]
    # distinct timestamps only: drop the planted ties
    tau = torch.cumsum(torch.ones_like(tau) * 0.5 + torch.arange(tau.shape[1]) * 1e-3, 1)
    ref = oracle.time_aware_interp(V, M, tau)
    prev, nxt, cur = oracle.interp_neighbors_time(M, tau, tau, 10, 128)
    vh = oracle.interp_gather(V, tau, tau, prev, nxt, cur)
    assert torch.equal(vh, ref)


def test_interp_step_sequence():
    g = load_golden("interp_step_seq")
    h = g["h0"]
    for t in range(g["V"].shape[1]):
        vh, h = oracle.interp_ssm_step(g["V"], g["M"], g["tau"], g["Abar"], g["Bbar"], h, t)
        assert rel_err(vh, g["Vhat"][:, t]) < 1e-6
        assert rel_err(h, g["h_seq"][t]) < 1e-5


def test_interp_ssm_obs_grid():
    g = load_golden("interp_ssm_obsgrid")
    y, h, vh = oracle.interp_ssm(g["V"], g["M"], g["tau"], g["A_log"], g["B"], g["C"], g["dt"],
                                 return_vhat=True)
    assert rel_err(vh, g["Vhat"]) < 1e-6
    assert rel_err(y, g["y"]) < TOL_FP32
    assert rel_err(h, g["h_last"]) < TOL_FP32


def test_streaming_inplace():
    for dtn, bf in (("fp32", False), ("bf16", True)):
        g = load_golden("stream_inplace_" + dtn)
        h, y = oracle.streaming_ssm_inplace(g["vhat"], g["h_in"], g["Abar"], g["Bbar"], g["C"],
                                            g["D"], bf16=bf)
        tol = 1e-6 if not bf else 1e-2
        assert rel_err(h, g["h_out"]) < tol
        assert rel_err(y, g["y"]) < tol


def test_streaming_step_composed():
    g = load_golden("stream_step_composed")
    h = g["h0"]
    for s in range(g["x"].shape[0]):
        h, y = oracle.streaming_step(g["x"][s], g["dt"][s], h, g["A_log"], g["B"][s], g["C"][s], g["D"])
        assert rel_err(y, g["y"][s]) < TOL_FP32
    assert rel_err(h, g["h_final"]) < TOL_FP32


def test_ring_stream():
    g = load_golden("ring_stream")
    rV, rM, rT, rH, h = (g[k].clone() for k in ("ring_V", "ring_M", "ring_tau", "ring_head", "h0"))
    for e in range(g["v"].shape[0]):
        y = oracle.ring_interp_then_ssm(rV, rM, rT, rH, g["v"][e], g["m"][e], g["tau"][e], h,
                                        g["Abar"], g["Bbar"], g["C"][e], g["D"], BLOCK_H=32)
        assert rel_err(y, g["y"][e]) < 1e-6
        assert rel_err(h, g["h"][e]) < 1e-6
    assert torch.equal(rH, g["ring_head_final"])
    assert torch.equal(rV, g["ring_V_final"])


def test_ssm_backward():
    g = load_golden("ssm_backward")
    du, dA, dB, dC = oracle.ssm_backward(g["u"], g["A"], g["B"], g["C"], g["h"], g["dY"])
    for a, k in ((du, "du"), (dA, "dA"), (dB, "dB"), (dC, "dC")):
        assert rel_err(a, g[k]) < TOL_FP32, k


def test_discretize_bwd():
    g = load_golden("discretize_bwd")
    dA, dB, ddt = oracle.zoh_discretize_bwd(g["A_log"], g["B"], g["dt"], g["Abar"], g["dAbar"], g["dBbar"])
    assert rel_err(dA, g["dA_log"]) < TOL_FP32
    assert rel_err(dB, g["dB"]) < TOL_FP32
    assert rel_err(ddt, g["ddt"]) < TOL_FP32


def test_dt_project_softplus_restatement():
    """The restated projection (the reference kernel does not compile): the
    softplus is log(1 + exp(x)) as written there, a large pre-activation
    overflows to inf and clamps to DT_MAX, and per-channel discretisation with
    a dt that is constant over H equals the reference's shared-dt discretisation."""
    g = torch.Generator().manual_seed(0)
    dt_raw = torch.randn(2, 5, 3, generator=g)
    W = torch.randn(3, 7, generator=g)
    bias = torch.randn(7, generator=g)
    dt = oracle.dt_project_softplus(dt_raw, W, bias, 1e-3, 0.5)
    acc = dt_raw @ W + bias
    assert torch.allclose(dt, torch.clamp(torch.nn.functional.softplus(acc), 1e-3, 0.5), rtol=1e-6, atol=1e-7)
    big = oracle.dt_project_softplus(dt_raw * 1e4, W, bias, 1e-3, 0.5)
    assert torch.isfinite(big).all() and float(big.max()) == 0.5
    A_log = torch.log(torch.empty(7).uniform_(0.5, 16, generator=g))
    B = torch.randn(2, 5, 7, generator=g)
    dts = torch.rand(2, 5, generator=g)
    a1, b1 = oracle.zoh_discretize_dt(A_log, B, dts[..., None].expand(2, 5, 7))
    a2, b2 = oracle.zoh_discretize(A_log, B, dts)
    assert torch.equal(a1, a2) and torch.equal(b1, b2)
