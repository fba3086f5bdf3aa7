"""GPU parity of the backward passes (ssm_backward, zoh_discretize_bwd) against
the golden fixtures minted from the reference and the CPU oracle on the same
seeded inputs."""
import pytest
import torch

import oracle
from conftest import TOL_BF16, TOL_FP32, load_golden, rel_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def cu(t):
    return t.to(dev)


def _scan_inputs(Bt, L, H, seed, dty=torch.float32):
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(Bt, L, H, generator=g)
    A = torch.empty(Bt, L, H).uniform_(0.5, 0.999, generator=g)
    B = torch.randn(Bt, L, H, generator=g) * 0.5
    C = torch.randn(Bt, L, H, generator=g)
    D = torch.randn(H, generator=g)
    dY = torch.randn(Bt, L, H, generator=g)
    _, h = oracle.ssm_forward(u, A, B, C, D)
    return [t.to(dty) for t in (u, A, B, C, h, dY)]


def test_ssm_backward_golden(cuda_ops):
    g = load_golden("ssm_backward")
    out = cuda_ops.ssm_backward(*(cu(g[k]) for k in ("u", "A", "B", "C", "h", "dY")))
    for name, t in zip(("du", "dA", "dB", "dC"), out):
        assert rel_err(t, g[name]) < TOL_FP32, name


@pytest.mark.parametrize("Bt,L,H", [(1, 1, 1), (2, 33, 37), (3, 257, 64), (2, 1000, 96), (1, 4099, 33),
                                    # 16-byte row pitch (TMA-staged kernel): one step, one exact
                                    # 64-step tile with a partial channel tile, a tile edge plus one
                                    (1, 1, 4), (2, 64, 36), (1, 129, 32)])
def test_ssm_backward_vs_oracle(cuda_ops, Bt, L, H):
    ins = _scan_inputs(Bt, L, H, seed=L * 31 + H)
    out = cuda_ops.ssm_backward(*(cu(t) for t in ins))
    ref = oracle.ssm_backward(*ins)
    for name, t, r in zip(("du", "dA", "dB", "dC"), out, ref):
        assert t.shape == r.shape
        assert rel_err(t, r) < TOL_FP32, name


def test_ssm_backward_bf16(cuda_ops):
    ins = _scan_inputs(2, 300, 64, seed=5, dty=torch.bfloat16)
    out = cuda_ops.ssm_backward(*(cu(t) for t in ins))
    ref = oracle.ssm_backward(*(t.float() for t in ins))
    for name, t, r in zip(("du", "dA", "dB", "dC"), out, ref):
        assert t.dtype == torch.bfloat16
        assert rel_err(t.float(), r) < TOL_BF16, name


def test_ssm_backward_matches_autograd(cuda_ops):
    """The reference's state-path gradients equal torch autograd of the forward
    recurrence with D held constant (f64 on the CPU)."""
    Bt, L, H = 2, 70, 8
    ins = _scan_inputs(Bt, L, H, seed=9)
    u, A, B, C, _, dY = (t.double().requires_grad_(True) for t in ins)
    hs, hcur = [], torch.zeros(Bt, H, dtype=torch.float64)
    for t in range(L):
        hcur = A[:, t] * hcur + B[:, t] * u[:, t]
        hs.append(hcur)
    y = C * torch.stack(hs, 1)       # D*u is a constant offset on the state path
    (y * dY.detach()).sum().backward()
    h = torch.stack(hs, 1).detach()
    out = cuda_ops.ssm_backward(*(cu(t.detach().float()) for t in (u, A, B, C)), cu(h.float()),
                                cu(dY.detach().float()))
    for name, t, r in zip(("du", "dA", "dB", "dC"), out, (u.grad, A.grad, B.grad, C.grad)):
        assert rel_err(t, r) < TOL_FP32, name


def test_ssm_backward_rejects_bad_args(cuda_ops):
    x = torch.zeros(2, 3, 4, device=dev)
    with pytest.raises(ValueError):
        cuda_ops.ssm_backward(x, x, x, x, x, x.double())
    with pytest.raises(ValueError):
        cuda_ops.ssm_backward(x, x, x, x, x, x[:, :2])
    with pytest.raises(ValueError):
        cuda_ops.ssm_backward(x.cpu(), x, x, x, x, x)
    e = torch.zeros(0, 3, 4, device=dev)
    assert cuda_ops.ssm_backward(e, e, e, e, e, e)[0].numel() == 0


def _disc_inputs(Bt, T, H, seed):
    g = torch.Generator().manual_seed(seed)
    A_log = torch.log(torch.empty(H).uniform_(0.5, 16, generator=g))
    B = torch.randn(Bt, T, H, generator=g)
    dt = torch.empty(Bt, T).exponential_(1.0, generator=g).clamp_(1e-6, 10)
    dt[0, 0] = 1e-7          # the |x| <= 1e-5 branch of the guarded expm1
    Abar, _ = oracle.zoh_discretize(A_log, B, dt)
    dAbar = torch.randn(Bt, T, H, generator=g)
    dBbar = torch.randn(Bt, T, H, generator=g)
    return A_log, B, dt, Abar, dAbar, dBbar


def test_discretize_bwd_golden(cuda_ops):
    g = load_golden("discretize_bwd")
    dA, dB, ddt = cuda_ops.zoh_discretize_bwd(*(cu(g[k]) for k in ("A_log", "B", "dt", "Abar", "dAbar", "dBbar")))
    assert rel_err(dA, g["dA_log"]) < TOL_FP32
    assert rel_err(dB, g["dB"]) < TOL_FP32
    # the reference's ddt is only the full sum over H when H fits one block, as in the golden
    assert rel_err(ddt, g["ddt"]) < TOL_FP32


@pytest.mark.parametrize("Bt,T,H", [(1, 1, 1), (2, 17, 37), (3, 33, 1024), (2, 50, 1500), (1, 40, 4100)])
def test_discretize_bwd_vs_oracle(cuda_ops, Bt, T, H):
    ins = _disc_inputs(Bt, T, H, seed=H + T)
    dA, dB, ddt = cuda_ops.zoh_discretize_bwd(*(cu(t) for t in ins))
    rA, rB, rdt = oracle.zoh_discretize_bwd(*ins)
    assert rel_err(dA, rA) < TOL_FP32
    assert rel_err(dB, rB) < TOL_FP32
    assert rel_err(ddt, rdt) < TOL_FP32


def test_discretize_bwd_repeated_calls_do_not_accumulate(cuda_ops):
    ins = [cu(t) for t in _disc_inputs(2, 20, 64, seed=3)]
    a1 = cuda_ops.zoh_discretize_bwd(*ins)[0].clone()
    a2 = cuda_ops.zoh_discretize_bwd(*ins)[0]
    assert rel_err(a2, a1) < 1e-6
