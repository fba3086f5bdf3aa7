"""GPU: chaining sequence slices with ssd_carry_fixup reproduces the
whole-sequence scan (ranks emulated as slices on one device)."""
import pytest
import torch

import oracle
from conftest import TOL_BF16, rel_err
from test_gpu_ssd import make_inputs

pytestmark = pytest.mark.gpu
dev = "cuda"


@pytest.mark.parametrize("N,R,L", [(64, 3, 700), (128, 4, 520), (64, 2, 64)])
def test_slices_chained_equal_whole_sequence(cuda_ops, N, R, L):
    x, dt, A_log, B, C, D = make_inputs(2, L, 3, 64, N, seed=N + R, dt_lo=1e-3)
    xd, dtd, Ad, Bd, Cd, Dd = (t.to(dev) for t in (x, dt, A_log, B, C, D))
    whole = cuda_ops.multihead_ssm(xd, Ad, Bd, Cd, dtd, Dd)
    from triton_ssm_b200 import parallel
    cuts = [parallel.shard_range(L, r, R) for r in range(R)]
    outs, Ss, ds = [], [], []
    for a, b in cuts:
        y, S, d = cuda_ops.multihead_ssm(xd[:, a:b].contiguous(), Ad, Bd[:, a:b].contiguous(),
                                         Cd[:, a:b].contiguous(), dtd[:, a:b].contiguous(), Dd,
                                         return_state=True, return_decay=True)
        outs.append(y)
        Ss.append(S)
        ds.append(d)
    S_all = torch.stack(Ss).contiguous()
    d_all = torch.stack(ds).contiguous()
    for r, (a, b) in enumerate(cuts):
        cuda_ops.ssd_carry_fixup(S_all, d_all, r, Cd[:, a:b].contiguous(), dtd[:, a:b].contiguous(), Ad, outs[r])
    cuda_ops.check_device_status()
    y = torch.cat(outs, dim=1)
    ref, _ = oracle.ssd_scan_chunked(x, dt, A_log, B, C, D, chunk=128)
    assert rel_err(y, ref) < TOL_BF16
    assert rel_err(y, whole) < TOL_BF16


def test_decay_output_matches_dt_sum(cuda_ops):
    x, dt, A_log, B, C, D = make_inputs(2, 333, 4, 64, 64, seed=1)
    _, _, d = cuda_ops.multihead_ssm(x.to(dev), A_log.to(dev), B.to(dev), C.to(dev), dt.to(dev), D.to(dev),
                                     return_state=True, return_decay=True)
    ref = dt.sum(1) * (-torch.exp(A_log)) * 1.4426950408889634
    assert rel_err(d, ref) < 1e-5


@pytest.mark.parametrize("Bt,L,H,N,K", [(2, 4096, 3, 64, 4), (1, 2048, 2, 128, 2), (1, 8192, 2, 64, 8)])
def test_in_device_pieces_equal_whole_sequence(cuda_ops, Bt, L, H, N, K):
    """Scanning each sequence as K pieces at once and chaining them with the
    pieces fix-up gives the whole-sequence outputs, final state and decay."""
    x, dt, A_log, B, C, D = make_inputs(Bt, L, H, 64, N, seed=L + K, dt_lo=1e-3)
    args = [t.to(dev) for t in (x, A_log, B, C, dt, D)]
    y1, h1, d1 = cuda_ops.multihead_ssm(*args, return_state=True, return_decay=True)
    yk, hk, dk = cuda_ops.multihead_ssm(*args, return_state=True, return_decay=True, pieces=K)
    cuda_ops.check_device_status()
    assert rel_err(yk, y1) < TOL_BF16
    assert rel_err(hk, h1) < 1e-4
    assert rel_err(dk, d1) < 1e-5
    ref, _ = oracle.ssd_scan_chunked(x, dt, A_log, B, C, D, chunk=128)
    assert rel_err(yk, ref) < TOL_BF16


def test_in_device_pieces_rejects_bad_split(cuda_ops):
    x, dt, A_log, B, C, D = make_inputs(1, 1000, 2, 64, 64, seed=3)
    with pytest.raises(ValueError):
        cuda_ops.multihead_ssm(*(t.to(dev) for t in (x, A_log, B, C, dt, D)), pieces=4)
