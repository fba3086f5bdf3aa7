"""Diagonal linear-recurrence scans, restated from ``ssm_scan.py`` (test oracle only)."""
import torch

from .discretize import expm1_ref


def ssm_forward(u, A, B, C, D, dtype=torch.float32):
    """``ssm_forward`` (``ssm_scan.py:239-264``) as a plain sequential recurrence.

    u, A, B, C [Bt,L,H]; D [H].  h_t = A_t*h_{t-1} + B_t*u_t with h_{-1} = 0
    (the (a, x) combine of ``:12-14`` applied left to right), y_t = C_t*h_t + D*u_t
    (``:116-124``).  Returns (y, h) [Bt,L,H] in ``dtype``.
    """
    u, A, B, C, D = (t.to(dtype) for t in (u, A, B, C, D))
    Bt, L, H = u.shape
    h = torch.zeros(Bt, H, dtype=dtype)
    hs = torch.empty(Bt, L, H, dtype=dtype)
    bu = B * u
    for t in range(L):
        h = A[:, t] * h + bu[:, t]
        hs[:, t] = h
    y = C * hs + D * u
    return y, hs


def ssm_backward(u, A, B, C, h, dY, dtype=torch.float32):
    """``ssm_backward`` (``ssm_scan.py:267-289``): reverse scan of dH.

    dH_t = C_t*dY_t + A_{t+1}*dH_{t+1} (``:142-166``); du = B*dH, dB = u*dH,
    dC = dY*h, dA_t = h_{t-1}*dH_t (``:216-231``).  D is treated as a constant,
    as in the reference (no dD).
    """
    u, A, B, C, h, dY = (t.to(dtype) for t in (u, A, B, C, h, dY))
    Bt, L, H = u.shape
    dH = torch.empty_like(u)
    acc = torch.zeros(Bt, H, dtype=dtype)
    for t in range(L - 1, -1, -1):
        a_next = A[:, t + 1] if t + 1 < L else torch.zeros(Bt, H, dtype=dtype)
        acc = a_next * acc + C[:, t] * dY[:, t]
        dH[:, t] = acc
    h_prev = torch.cat([torch.zeros(Bt, 1, H, dtype=dtype), h[:, :-1]], dim=1)
    return B * dH, h_prev * dH, u * dH, dY * h


def selective_scan(x, dt, A_log, B, C, D, h0=None, dtype=torch.float32, variant="fp32"):
    """The config-1 pipeline ``zoh_discretize`` → ``ssm_forward`` over the
    flattened channel axis H' = D*N with the readout summed over N.

    x [Bt,L,D]; dt [Bt,L]; A_log [D,N]; B, C [Bt,L,N]; D [D].  Per (b,d,n):
    Abar = exp(dt*a), Bbar = expm1_ref(dt*a)/(a+1e-12)*B[b,t,n]
    (``discretize_kernel.py:38-54``), h = Abar*h + Bbar*x[b,t,d]
    (``ssm_scan.py:36-45``), y[b,t,d] = sum_n C[b,t,n]*h[d,n] + D[d]*x[b,t,d]
    (``ssm_scan.py:116-124`` plus the host-side sum over N).
    Returns (y [Bt,L,D], h_last [Bt,D,N]).
    """
    x, dt, A_log, B, C, D = (t.to(dtype) for t in (x, dt, A_log, B, C, D))
    Bt, L, Dd = x.shape
    N = A_log.shape[1]
    a = -torch.exp(A_log)                                # [D,N]
    h = torch.zeros(Bt, Dd, N, dtype=dtype) if h0 is None else h0.to(dtype).clone()
    y = torch.empty(Bt, L, Dd, dtype=dtype)
    for t in range(L):
        xx = dt[:, t, None, None] * a                    # [Bt,D,N]
        Abar = torch.exp(xx)
        Bbar = expm1_ref(xx, variant) / (a + 1e-12) * B[:, t, None, :]
        h = Abar * h + Bbar * x[:, t, :, None]
        y[:, t] = (h * C[:, t, None, :]).sum(-1) + D * x[:, t]
    return y, h
