"""GPU parity of the race-free ring-buffer streaming step
(streaming_inference_kernel.py:74-156) against the golden minted from the
reference and the CPU oracle, and the checkpoint / restore of long-running
streams."""
import pytest
import torch

import oracle
from conftest import load_golden, rel_err

pytestmark = pytest.mark.gpu
dev = "cuda"


def cu(t):
    return t.to(dev)


def test_ring_stream_golden(cuda_ops):
    g = load_golden("ring_stream")
    rV, rM, rT, rH, h = (cu(g[k].clone()) for k in ("ring_V", "ring_M", "ring_tau", "ring_head", "h0"))
    for e in range(g["v"].shape[0]):
        y = cuda_ops.streaming_interp_then_ssm(rV, rM, rT, rH, cu(g["v"][e]), cu(g["m"][e]), cu(g["tau"][e]), h,
                                               cu(g["Abar"]), cu(g["Bbar"]), cu(g["C"][e]), cu(g["D"]), BLOCK_H=32)
        assert rel_err(y, g["y"][e]) < 1e-6, e
        assert rel_err(h, g["h"][e]) < 1e-6, e
    assert torch.equal(rH.cpu(), g["ring_head_final"])
    assert torch.equal(rV.cpu(), g["ring_V_final"])
    assert torch.equal(rM.cpu(), g["ring_M_final"])
    assert torch.equal(rT.cpu(), g["ring_tau_final"])


def _events(Bt, H, n, seed, p_obs=0.7, p_tile_gap=0.3, tile=32):
    """Masks with whole tiles missing in some events, so the backward search
    has to look several slots deep."""
    g = torch.Generator().manual_seed(seed)
    ev = []
    for _ in range(n):
        m = (torch.rand(Bt, H, generator=g) < p_obs).float()
        nt = (H + tile - 1) // tile
        gap = torch.rand(Bt, nt, generator=g) < p_tile_gap
        for b in range(Bt):
            for t in range(nt):
                if gap[b, t]:
                    m[b, t * tile:(t + 1) * tile] = 0.0
        ev.append(dict(v=torch.randn(Bt, H, generator=g), m=m, tau=torch.rand(Bt, generator=g),
                       C=torch.randn(Bt, H, generator=g)))
    return ev


@pytest.mark.parametrize("Bt,H,K,BLOCK_H", [(3, 300, 4, 32), (2, 1000, 10, 128), (4, 70, 2, 16), (2, 129, 0, 64),
                                            (1, 256, 7, 1)])
def test_ring_vs_oracle(cuda_ops, Bt, H, K, BLOCK_H):
    g = torch.Generator().manual_seed(H + K)
    KR = K + 1
    Abar = torch.rand(H, generator=g) * 0.5 + 0.45
    Bbar = torch.randn(H, generator=g) * 0.3
    D = torch.randn(H, generator=g)
    ring = [torch.zeros(Bt, KR, H), torch.zeros(Bt, KR, H), torch.zeros(Bt, KR),
            torch.randint(0, KR, (Bt,), generator=g, dtype=torch.int32)]
    h = torch.randn(Bt, H, generator=g)
    dring = [cu(t.clone()) for t in ring]
    dh = cu(h.clone())
    for e, ev in enumerate(_events(Bt, H, 3 * KR + 2, seed=K * 7 + H, tile=max(BLOCK_H, 8))):
        y_ref = oracle.ring_interp_then_ssm(*ring, ev["v"], ev["m"], ev["tau"], h, Abar, Bbar, ev["C"], D,
                                            BLOCK_H=BLOCK_H)
        y = cuda_ops.streaming_interp_then_ssm(*dring, cu(ev["v"]), cu(ev["m"]), cu(ev["tau"]), dh, cu(Abar),
                                               cu(Bbar), cu(ev["C"]), cu(D), BLOCK_H=BLOCK_H)
        assert rel_err(y, y_ref) < 1e-6, e
        assert rel_err(dh, h) < 1e-6, e
        for a, r in zip(dring, ring):
            assert torch.equal(a.cpu(), r), e


def test_ring_rejects_bad_args(cuda_ops):
    Bt, H, KR = 2, 8, 3
    z = lambda *s: torch.zeros(*s, device=dev)
    args = [z(Bt, KR, H), z(Bt, KR, H), z(Bt, KR), torch.zeros(Bt, dtype=torch.int32, device=dev), z(Bt, H),
            z(Bt, H), z(Bt), z(Bt, H), z(H), z(H), z(Bt, H), z(H)]
    bad = list(args)
    bad[3] = torch.zeros(Bt, dtype=torch.int64, device=dev)
    with pytest.raises(ValueError):
        cuda_ops.streaming_interp_then_ssm(*bad)
    bad = list(args)
    bad[4] = z(Bt, H + 1)
    with pytest.raises(ValueError):
        cuda_ops.streaming_interp_then_ssm(*bad)
    bad = list(args)
    bad[7] = z(H, Bt).t()
    with pytest.raises(ValueError):
        cuda_ops.streaming_interp_then_ssm(*bad)


def test_streaming_ring_checkpoint_restore(cuda_ops, tmp_path):
    Bt, H, K = 3, 256, 5
    g = torch.Generator().manual_seed(4)
    ring = cuda_ops.StreamingRing(Bt, H, K, torch.rand(H, generator=g) * 0.9, torch.randn(H, generator=g),
                                  torch.randn(H, generator=g), device=dev, block_h=32)
    evs = _events(Bt, H, 12, seed=8)
    for ev in evs[:5]:
        ring.step(cu(ev["v"]), cu(ev["m"]), cu(ev["tau"]), cu(ev["C"]))
    ck = ring.checkpoint()
    path = tmp_path / "streams.pt"
    ring.save(path)
    first = [ring.step(cu(ev["v"]), cu(ev["m"]), cu(ev["tau"]), cu(ev["C"])).clone() for ev in evs[5:]]
    h_first = ring.h.clone()
    ring.restore(ck)
    assert ring.steps == 5
    second = [ring.step(cu(ev["v"]), cu(ev["m"]), cu(ev["tau"]), cu(ev["C"])).clone() for ev in evs[5:]]
    for a, b in zip(first, second):
        assert torch.equal(a, b)
    assert torch.equal(ring.h, h_first)
    again = cuda_ops.StreamingRing.load(path, device=dev)
    third = [again.step(cu(ev["v"]), cu(ev["m"]), cu(ev["tau"]), cu(ev["C"])).clone() for ev in evs[5:]]
    for a, b in zip(first, third):
        assert torch.equal(a, b)
    with pytest.raises(ValueError):
        cuda_ops.StreamingRing(Bt, H, K + 1, ring.Abar, ring.Bbar, ring.D, block_h=32).restore(ck)
