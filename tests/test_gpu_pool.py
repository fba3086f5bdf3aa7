"""GPU parity of the mean-pooled logit head (streaming_inference_kernel.py:
159-194), standalone and fused into the scan's epilogue, against the CPU
oracle.  The reference kernel does not run, so the oracle's restatement is the
only pin for this function."""
import pytest
import torch

import oracle
from conftest import TOL_BF16, TOL_FP32, rel_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def cu(t):
    return t.to(dev)


@pytest.mark.parametrize("Bt,T,H", [(1, 1, 1), (3, 33, 37), (2, 100, 1024), (4, 1024, 64), (2, 5, 4099)])
def test_mean_pool_logit_vs_oracle(cuda_ops, Bt, T, H):
    g = torch.Generator().manual_seed(T + H)
    x = torch.randn(Bt, T, H, generator=g)
    W = torch.randn(H, generator=g)
    bias = torch.randn(1, generator=g)
    out = cuda_ops.mean_pool_logit(cu(x), cu(W), cu(bias))
    ref = oracle.mean_pool_logit(x, W, bias)
    assert out.shape == (Bt,)
    assert (out.cpu() - ref).abs().max() < 1e-5 * (1 + ref.abs().max())
    outb = cuda_ops.mean_pool_logit(cu(x.bfloat16()), cu(W), cu(bias))
    refb = oracle.mean_pool_logit(x.bfloat16().float(), W, bias)
    assert (outb.cpu() - refb).abs().max() < 1e-5 * (1 + refb.abs().max())


def test_mean_pool_logit_empty_is_bias(cuda_ops):
    b = torch.tensor([0.25], device=dev)
    out = cuda_ops.mean_pool_logit(torch.zeros(3, 0, 8, device=dev), torch.ones(8, device=dev), b)
    assert torch.equal(out.cpu(), torch.full((3,), 0.25))


@pytest.mark.parametrize("dty", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("Bt,L,H", [(2, 300, 64), (3, 1000, 96), (1, 17, 5)])
def test_ssm_forward_fused_pool(cuda_ops, dty, Bt, L, H):
    g = torch.Generator().manual_seed(L * 3 + H)
    u = torch.randn(Bt, L, H, generator=g)
    A = torch.empty(Bt, L, H).uniform_(0.5, 0.99, generator=g)
    B = torch.randn(Bt, L, H, generator=g) * 0.5
    C = torch.randn(Bt, L, H, generator=g)
    D = torch.randn(H, generator=g)
    W = torch.randn(H, generator=g)
    bias = torch.randn(1, generator=g)
    ins = [cu(t.to(dty)) for t in (u, A, B, C, D)]
    y, h, logits = cuda_ops.ssm_forward(*ins, pool=(cu(W), cu(bias)))
    y2, h2 = cuda_ops.ssm_forward(*ins)
    # where rows are not TMA-addressable (H=5) the pooled variant splits the sequence
    # into shorter per-warp runs, so the scan's float association (not its math)
    # differs from the plain kernel there
    tol = 1e-5 if dty == torch.float32 else 1e-2
    assert rel_err(y.float(), y2.float()) < tol and rel_err(h.float(), h2.float()) < tol
    ref = oracle.mean_pool_logit(y.float().cpu(), W, bias)     # pooling what the output holds
    assert (logits.cpu() - ref).abs().max() < 1e-5 * (1 + ref.abs().max())
    ry, _ = oracle.ssm_forward(*(t.to(dty).float() for t in (u, A, B, C, D)))
    assert rel_err(y.float(), ry) < (TOL_FP32 if dty == torch.float32 else TOL_BF16)
