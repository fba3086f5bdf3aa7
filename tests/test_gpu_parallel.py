"""GPU: chaining sequence slices with ssd_carry_fixup reproduces the
whole-sequence scan (ranks emulated as slices on one device)."""
import pytest
import torch

import oracle
from conftest import TOL_BF16, parity, rel_err
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


@pytest.mark.parametrize("N", [64, 128])
def test_slices_chained_slow_decay(cuda_ops, N):
    """A decay slow enough that a slice's carry reaches far more than the 16
    chunks the fix-up spreads over CTAs (dt = 2e-3, A = -0.5: ~100k tokens to
    underflow): the last CTA walks the rest of each slice, in both the
    cross-slice and the in-device pieces fix-ups."""
    Bt, L, H, P, R = 1, 6144, 2, 64, 2
    x, dt, A_log, B, C, D = make_inputs(Bt, L, H, P, N, seed=5)
    dt = torch.full_like(dt, 2e-3)
    A_log = torch.full_like(A_log, float(torch.log(torch.tensor(0.5))))
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
    yk = cuda_ops.multihead_ssm(xd, Ad, Bd, Cd, dtd, Dd, pieces=2)
    cuda_ops.check_device_status()
    y = torch.cat(outs, dim=1)
    ref, _ = oracle.ssd_scan_chunked(x, dt, A_log, B, C, D, chunk=128)
    parity("slow-decay slices chained (N%d, 2 x 3072 tokens)" % N, y, ref, TOL_BF16)
    assert rel_err(y, whole) < TOL_BF16
    assert rel_err(yk, ref) < TOL_BF16 and rel_err(yk, whole) < TOL_BF16


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


@pytest.mark.parametrize("R,K,L", [(8, 8, 131072), (2, 8, 262144)])
def test_config4_sharded_length(cuda_ops, R, K, L):
    """Config 4's chain at the lengths the bench shards: B1 H4 P64 N128 bf16,
    A_h = -(1 + h mod 16), a sequence of L tokens as R rank slices (emulated on
    one GPU), each scanned as K in-device pieces.  Each slice writes its final
    state and decay straight into its row of one packed buffer, as the bench's
    all-gather lays them out; ssd_carry_fixup_packed then chains the slices.
    (8 x 8 over 131,072 tokens; 2 x 8 over 262,144 = the 131,072-token slice
    each of 8 ranks holds in the bench, chained to the slice before it.)
    Reference semantics: the carry scan of ssm_scan.py:53-98 lifted to slices."""
    from triton_ssm_b200 import workloads
    Bt, H, P, N = 1, 4, 64, 128
    inp = workloads.ssd_inputs_slice(Bt, 0, L, H, P, N, "cpu", seed=4)
    A, D = inp["A_log"].to(dev), inp["D"].to(dev)
    n, m = Bt * H * P * N, Bt * H
    packed = torch.empty(R, n + m, device=dev)
    Ls = L // R
    slices = []
    for r in range(R):
        sl = slice(r * Ls, (r + 1) * Ls)
        x, dt, Bm, Cm = (inp[k][:, sl].contiguous().to(dev) for k in ("x", "dt", "B", "C"))
        y, _, _ = cuda_ops.multihead_ssm(x, A, Bm, Cm, dt, D, return_state=True, return_decay=True, pieces=K,
                                         state_out=packed[r, :n].view(Bt, H, P, N),
                                         decay_out=packed[r, n:].view(Bt, H))
        slices.append((y, Cm, dt))
    for r, (y, Cm, dt) in enumerate(slices):
        cuda_ops.ssd_carry_fixup_packed(packed, r, Cm, dt, A, y)
    cuda_ops.check_device_status()
    y = torch.cat([t[0] for t in slices], dim=1)
    ref, href = oracle.ssd_scan_chunked(inp["x"], inp["dt"], inp["A_log"], inp["B"], inp["C"], inp["D"], chunk=256)
    parity("config 4 y, %d slices x %d pieces, L=%d (B1 H4 N128, bf16)" % (R, K, L), y, ref, TOL_BF16)
    # the last slice's packed state chained over all slices is the whole sequence's final state
    carry = torch.zeros(Bt, H, P, N, device=dev)
    for r in range(R):
        carry = torch.exp2(packed[r, n:].view(Bt, H))[..., None, None] * carry + packed[r, :n].view(Bt, H, P, N)
    parity("config 4 final state chained over the %d slices" % R, carry, href, TOL_BF16)


def test_pieces_final_state_kernel(cuda_ops):
    """tssm_ssd_pieces_final_state chains the pieces' states in order and sums
    their log2 decays (checked against the same chain in torch)."""
    g = torch.Generator().manual_seed(2)
    Bt, K, H, P, N = 3, 4, 5, 8, 12
    S = torch.randn(Bt * K, H, P, N, generator=g).to(dev)
    d = (-torch.rand(Bt * K, H, generator=g) * 3).to(dev)
    from triton_ssm_b200 import _lib
    hl = torch.empty(Bt, H, P, N, device=dev)
    dl = torch.empty(Bt, H, device=dev)
    _lib.call("tssm_ssd_pieces_final_state", _lib.ptr(S), _lib.ptr(d), K, _lib.ptr(hl), _lib.ptr(dl), Bt, H, P, N,
              _lib.stream_of(S))
    Sv, dv = S.view(Bt, K, H, P, N), d.view(Bt, K, H)
    ref = Sv[:, 0].clone()
    for k in range(1, K):
        ref = torch.exp2(dv[:, k])[..., None, None] * ref + Sv[:, k]
    assert rel_err(hl, ref) < 1e-6
    assert rel_err(dl, dv.sum(1)) < 1e-6
