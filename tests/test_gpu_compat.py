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
