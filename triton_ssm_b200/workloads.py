"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset is involved; these ARE the workloads).

Every generator takes a device and a seed and builds the tensors there with a
torch.Generator, so a rank can make its own shard without any exchange.
"""
import math

import torch

# Config 2 (multi-head chunked scan)
C2 = dict(Bt=16, H=8, P=64, N=64, L=8192, chunk=256)
# Config 5 (streaming)
C5 = dict(S=4096, H=16, P=64, N=64)
# Config 3 (fused interpolation + SSM)
C3 = dict(Bt=32, T=2048, Lq=4096, D=256, N=16)
# Config 1 (discretize + selective scan)
C1 = dict(Bt=4, L=1024, D=64, N=16)
# Config 4 (sequence-parallel scan)
C4 = dict(Bt=4, H=32, P=64, N=128, L=1048576)


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    return g


def ssd_inputs(Bt, L, H, P, N, device, seed, dt_range=(1e-3, 1.0)):
    """x, B, C bf16 ~ N(0,1) (B, C scaled 1/sqrt(N)); dt log-uniform on dt_range
    per (b,t,h); A_h = -exp(U(log 0.5, log 16)) per head (A_log = log(-A_h));
    D ~ N(0,1)."""
    g = _gen(device, seed)
    x = torch.randn(Bt, L, H * P, device=device, generator=g).to(torch.bfloat16)
    lo, hi = math.log(dt_range[0]), math.log(dt_range[1])
    dt = torch.exp(torch.empty(Bt, L, H, device=device).uniform_(lo, hi, generator=g))
    A_log = torch.empty(H, device=device).uniform_(math.log(0.5), math.log(16.0), generator=g)
    s = 1.0 / math.sqrt(N)
    B = (torch.randn(Bt, L, H, N, device=device, generator=g) * s).to(torch.bfloat16)
    C = (torch.randn(Bt, L, H, N, device=device, generator=g) * s).to(torch.bfloat16)
    D = torch.randn(H * P, device=device, generator=g)
    return dict(x=x, dt=dt, A_log=A_log, B=B, C=C, D=D)


def ssd_bytes(Bt, L, H, P, N, with_state=False):
    """Compulsory HBM bytes of one multi-head SSD pass: read x, B, C (bf16),
    dt (f32), A_log, D (f32); write y (bf16) [+ final f32 state]."""
    b = 2 * Bt * L * H * P * 2 + 2 * Bt * L * H * N * 2 + Bt * L * H * 4 + H * 4 + H * P * 4
    if with_state:
        b += Bt * H * P * N * 4
    return b


def ssd_updates(Bt, L, H, P, N):
    return Bt * L * H * P * N


def stream_inputs(S, H, P, N, device, seed, nsets=16):
    """Config 5: f32 state [S,H,P,N] ~ N(0,1)*0.1, and `nsets` pre-generated
    event sets (x bf16 ~ N(0,1); dt ~ Exp(1) per stream; B, C bf16 scaled
    1/sqrt(N)) that the steps cycle through; A_log per head, D [H,P]."""
    g = _gen(device, seed)
    h = torch.randn(S, H, P, N, device=device, generator=g) * 0.1
    A_log = torch.empty(H, device=device).uniform_(math.log(0.5), math.log(16.0), generator=g)
    D = torch.randn(H, P, device=device, generator=g)
    s = 1.0 / math.sqrt(N)
    events = []
    for _ in range(nsets):
        events.append(dict(
            x=torch.randn(S, H, P, device=device, generator=g).to(torch.bfloat16),
            dt=torch.empty(S, device=device).exponential_(1.0, generator=g),
            B=(torch.randn(S, H, N, device=device, generator=g) * s).to(torch.bfloat16),
            C=(torch.randn(S, H, N, device=device, generator=g) * s).to(torch.bfloat16)))
    return dict(h=h, A_log=A_log, D=D, events=events)


def stream_bytes(S, H, P, N):
    return 2 * S * H * P * N * 4 + 2 * S * H * P * 2 + 2 * S * H * N * 2 + S * 4 + H * 4 + H * P * 4


def ssd_inputs_slice(Bt, L0, Ls, H, P, N, device, seed, block=1 << 14, A_mode="config1"):
    """The [L0, L0+Ls) slice of a long sequence (config 4), generated in blocks
    of `block` tokens each seeded by its index, so every rank can build its own
    slice and the slices of any rank count concatenate to the same sequence.
    A_h = -(1 + h mod 16) ("A as in config 1", per head); dt log-uniform on [1e-3, 1].
    """
    assert L0 % block == 0, "slices start on a block boundary"
    x = torch.empty(Bt, Ls, H * P, device=device, dtype=torch.bfloat16)
    dt = torch.empty(Bt, Ls, H, device=device)
    B = torch.empty(Bt, Ls, H, N, device=device, dtype=torch.bfloat16)
    C = torch.empty(Bt, Ls, H, N, device=device, dtype=torch.bfloat16)
    s = 1.0 / math.sqrt(N)
    for o in range(0, Ls, block):
        n = min(block, Ls - o)
        g = _gen(device, seed * 1000003 + (L0 + o) // block)
        x[:, o:o + n] = torch.randn(Bt, n, H * P, device=device, generator=g).to(torch.bfloat16)
        dt[:, o:o + n] = torch.exp(torch.empty(Bt, n, H, device=device).uniform_(math.log(1e-3), 0.0, generator=g))
        B[:, o:o + n] = (torch.randn(Bt, n, H, N, device=device, generator=g) * s).to(torch.bfloat16)
        C[:, o:o + n] = (torch.randn(Bt, n, H, N, device=device, generator=g) * s).to(torch.bfloat16)
    if A_mode == "config1":
        A_log = torch.log(1.0 + (torch.arange(H, device=device) % 16).float())
    else:
        A_log = torch.empty(H, device=device).uniform_(math.log(0.5), math.log(16.0), generator=_gen(device, seed))
    D = torch.randn(H * P, device=device, generator=_gen(device, seed + 1))
    return dict(x=x, dt=dt, A_log=A_log, B=B, C=C, D=D)
