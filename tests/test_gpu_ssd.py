"""GPU parity of the tcgen05 multi-head SSD scan against the CPU oracle (whose
semantics are pinned to the reference by tests/golden/ssd_composed.npz)."""
import pytest
import torch

import oracle
from conftest import TOL_BF16, parity, rel_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def make_inputs(Bt, L, H, P, N, seed, dt_lo=1e-3):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(Bt, L, H * P, generator=g).bfloat16()
    dt = torch.exp(torch.empty(Bt, L, H).uniform_(torch.log(torch.tensor(dt_lo)).item(), 0.0, generator=g))
    A_log = torch.empty(H).uniform_(torch.log(torch.tensor(0.5)).item(), torch.log(torch.tensor(16.0)).item(),
                                    generator=g)
    B = (torch.randn(Bt, L, H, N, generator=g) / N ** 0.5).bfloat16()
    C = (torch.randn(Bt, L, H, N, generator=g) / N ** 0.5).bfloat16()
    D = torch.randn(H * P, generator=g)
    return x, dt, A_log, B, C, D


def run(ts, x, dt, A_log, B, C, D, **kw):
    out = ts.multihead_ssm(x.to(dev), A_log.to(dev), B.to(dev), C.to(dev), dt.to(dev), D.to(dev), **kw)
    ts.check_device_status()
    return out


@pytest.mark.parametrize("L", [1, 64, 200])
@pytest.mark.parametrize("bdisc", ["euler", "zoh"])
def test_ssd_small_vs_oracle(cuda_ops, L, bdisc):
    x, dt, A_log, B, C, D = make_inputs(2, L, 3, 64, 64, seed=L)
    y, hl = run(cuda_ops, x, dt, A_log, B, C, D, bdisc=bdisc, return_state=True)
    ry, rh = oracle.ssd_scan(x, dt, A_log, B, C, D, bdisc=bdisc)
    assert y.dtype == torch.bfloat16 and y.shape == x.shape
    assert rel_err(y, ry) < TOL_BF16
    assert rel_err(hl, rh) < TOL_BF16


def test_ssd_n128_and_h0(cuda_ops):
    x, dt, A_log, B, C, D = make_inputs(1, 150, 2, 64, 128, seed=5)
    g = torch.Generator().manual_seed(9)
    h0 = torch.randn(1, 2, 64, 128, generator=g) * 0.3
    y, hl = run(cuda_ops, x, dt, A_log, B, C, D, h0=h0.to(dev), return_state=True)
    ry, rh = oracle.ssd_scan(x, dt, A_log, B, C, D, h0=h0)
    assert rel_err(y, ry) < TOL_BF16
    assert rel_err(hl, rh) < TOL_BF16


def test_ssd_slow_decay_long(cuda_ops):
    # small |A*dt| keeps the state alive across many chunks (carry path dominates)
    x, dt, A_log, B, C, D = make_inputs(1, 1000, 2, 64, 64, seed=11, dt_lo=1e-4)
    dt = dt * 0.01
    y, hl = run(cuda_ops, x, dt, A_log, B, C, D, return_state=True)
    ry, rh = oracle.ssd_scan_chunked(x, dt, A_log, B, C, D, chunk=100)
    assert rel_err(y, ry) < TOL_BF16
    assert rel_err(hl, rh) < TOL_BF16


def test_ssd_config2_full_size(cuda_ops):
    """Config 2 at full size (B16 H8 P64 N64 L8192) against the chunked oracle."""
    torch.set_num_threads(max(1, torch.get_num_threads()))
    x, dt, A_log, B, C, D = make_inputs(16, 8192, 8, 64, 64, seed=2)
    y, hl = run(cuda_ops, x, dt, A_log, B, C, D, return_state=True)
    ry, rh = oracle.ssd_scan_chunked(x, dt, A_log, B, C, D, chunk=256)
    parity("config 2 y  (B16 H8 P64 N64 L8192, bf16)", y, ry, TOL_BF16)
    parity("config 2 h_last (f32 state)", hl, rh, TOL_BF16)


def test_ssd_linearity_and_determinism(cuda_ops):
    x, dt, A_log, B, C, D = make_inputs(2, 300, 4, 64, 64, seed=3)
    x2 = make_inputs(2, 300, 4, 64, 64, seed=4)[0]
    ya = run(cuda_ops, x, dt, A_log, B, C, D).float()
    yb = run(cuda_ops, x2, dt, A_log, B, C, D).float()
    yab = run(cuda_ops, (x.float() + x2.float()).bfloat16(), dt, A_log, B, C, D).float()
    assert rel_err(yab, ya + yb) < 3 * TOL_BF16
    ya2 = run(cuda_ops, x, dt, A_log, B, C, D).float()
    assert torch.equal(ya, ya2)


def test_ssd_rejects_unsupported(cuda_ops):
    x, dt, A_log, B, C, D = make_inputs(1, 10, 2, 32, 64, seed=0)
    with pytest.raises(ValueError):
        run(cuda_ops, x, dt, A_log, B, C, D)


# ---------------------------------------------------------------- diagonal mode
def test_multihead_diag_golden(cuda_ops):
    from conftest import TOL_FP32, load_golden
    g = load_golden("mh_diag_composed")
    y = cuda_ops.multihead_ssm(g["x"].to(dev), g["A_log"].to(dev), g["B"].to(dev), g["C"].to(dev),
                               g["dt"].to(dev), g["D"].to(dev), mode="diag")
    assert rel_err(y, g["y"]) < TOL_FP32


@pytest.mark.parametrize("hd,L,dty,bdisc", [(64, 1000, torch.float32, "euler"), (33, 257, torch.float32, "zoh"),
                                            (128, 300, torch.bfloat16, "euler"), (8, 5, torch.float32, "euler")])
def test_multihead_diag_vs_oracle(cuda_ops, hd, L, dty, bdisc):
    from conftest import TOL_FP32
    gen = torch.Generator().manual_seed(hd + L)
    Bt, nh = 2, 3
    u = torch.randn(Bt, L, nh * hd, generator=gen).to(dty)
    A_log = torch.empty(nh, hd).uniform_(-0.7, 2.7, generator=gen)
    B = torch.randn(Bt, L, nh, hd, generator=gen).to(dty)
    C = torch.randn(Bt, L, nh, hd, generator=gen).to(dty)
    dt = torch.exp(torch.empty(Bt, L, nh).uniform_(-6.9, 0.0, generator=gen))
    D = torch.randn(nh * hd, generator=gen)
    y = cuda_ops.multihead_ssm(u.to(dev), A_log.to(dev), B.to(dev), C.to(dev), dt.to(dev), D.to(dev),
                               mode="diag", bdisc=bdisc)
    ry, _ = oracle.multihead_diag(u, A_log, B, C, dt, D, bdisc=bdisc)
    tol = TOL_FP32 if dty == torch.float32 else TOL_BF16
    assert y.dtype == dty and rel_err(y, ry) < tol
