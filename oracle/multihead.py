"""Multi-head scans (test oracle only).

Two state semantics, both restated from ``multihead_ssm_kernel.py``:

* ``multihead_diag`` — the reference's own diagonal state h[b,h,p]
  (``multihead_ssm_kernel.py:54-102`` local scan, ``:141-187`` combine and
  readout) with the kernel's compile errors (scalar indexing at ``:101``,
  item assignment at ``:151-152``) read as their evident intent.
* ``ssd_scan`` — the outer-product state h[b,h,p,n] that the config-2/4
  workload names (B*L*H*P*N state updates): per head a scalar decay
  exp(dt*A_h) (``:66-69``), the Euler input dt*B (``:73``) or the ZOH input of
  ``discretize_kernel.py:50-54``, and the readout y[p] = sum_n C[n]*h[p,n] +
  D[p]*x[p].  For every fixed (p, n) this is exactly ``ssm_scan.py``'s
  diagonal recurrence, which is how the golden fixture pins it.
"""
import torch

from .discretize import expm1_ref


def _input_coeff(dt, a, bdisc):
    """Per-(b,t,h) factor multiplying B: dt (Euler, ``multihead_ssm_kernel.py:73``)
    or expm1_ref(dt*a)/(a+1e-12) (ZOH, ``discretize_kernel.py:50-54``)."""
    if bdisc == "euler":
        return dt
    if bdisc == "zoh":
        return expm1_ref(dt * a, "fp32") / (a + 1e-12)
    raise ValueError(bdisc)


def ssd_scan(x, dt, A_log, B, C, D, bdisc="euler", h0=None, dtype=torch.float32):
    """Sequential outer-product scan.

    x [Bt,L,H*P]; dt [Bt,L,H]; A_log [H] (log(-A_h)); B, C [Bt,L,H,N]; D [H*P].
    Returns (y [Bt,L,H*P], h_last [Bt,H,P,N]).
    """
    x, dt, A_log, B, C, D = (t.to(dtype) for t in (x, dt, A_log, B, C, D))
    Bt, L, H, N = B.shape
    P = x.shape[2] // H
    xs = x.view(Bt, L, H, P)
    a = -torch.exp(A_log)                                  # [H]
    dA = torch.exp(dt * a)                                 # [Bt,L,H]
    beta = _input_coeff(dt, a, bdisc)                      # [Bt,L,H]
    h = torch.zeros(Bt, H, P, N, dtype=dtype) if h0 is None else h0.to(dtype).clone()
    y = torch.empty(Bt, L, H, P, dtype=dtype)
    for t in range(L):
        Bb = beta[:, t, :, None] * B[:, t]                 # [Bt,H,N]   (dt*B first, :73)
        h = dA[:, t, :, None, None] * h + xs[:, t, :, :, None] * Bb[:, :, None, :]
        y[:, t] = torch.einsum("bhpn,bhn->bhp", h, C[:, t]) + D.view(H, P) * xs[:, t]
    return y.reshape(Bt, L, H * P), h


def ssd_scan_chunked(x, dt, A_log, B, C, D, chunk=64, bdisc="euler", h0=None,
                     dtype=torch.float32, return_state=True):
    """The same recurrence in chunked (matrix) form — used for the large-size
    CPU baseline and to cross-check ``ssd_scan``.  Within a chunk with
    s_i = sum_{k<=i} dt_k*A_h:
        y_i = sum_{j<=i} exp(s_i - s_j)*beta_j*(C_i.B_j)*x_j + exp(s_i)*C_i.h_in + D*x_i
        h_out = exp(s_last)*h_in + sum_j exp(s_last - s_j)*beta_j*x_j (x) B_j
    """
    x, dt, A_log, B, C, D = (t.to(dtype) for t in (x, dt, A_log, B, C, D))
    Bt, L, H, N = B.shape
    P = x.shape[2] // H
    a = -torch.exp(A_log)
    beta = _input_coeff(dt, a, bdisc)                      # [Bt,L,H]
    h = torch.zeros(Bt, H, P, N, dtype=dtype) if h0 is None else h0.to(dtype).clone()
    y = torch.empty(Bt, L, H, P, dtype=dtype)
    xs = x.view(Bt, L, H, P)
    for c0 in range(0, L, chunk):
        c1 = min(L, c0 + chunk)
        Q = c1 - c0
        la = (dt[:, c0:c1] * a).permute(0, 2, 1)           # [Bt,H,Q]
        s = torch.cumsum(la, dim=-1)
        xc = xs[:, c0:c1].permute(0, 2, 1, 3)              # [Bt,H,Q,P]
        Bc = B[:, c0:c1].permute(0, 2, 1, 3)               # [Bt,H,Q,N]
        Cc = C[:, c0:c1].permute(0, 2, 1, 3)
        bc = beta[:, c0:c1].permute(0, 2, 1)               # [Bt,H,Q]
        diff = s[..., :, None] - s[..., None, :]           # [Bt,H,Q,Q]
        tri = torch.ones(Q, Q, dtype=torch.bool).tril()
        Lm = torch.where(tri, torch.exp(torch.where(tri, diff, torch.zeros((), dtype=dtype))),
                         torch.zeros((), dtype=dtype))
        G = Cc @ Bc.transpose(-1, -2)                      # [Bt,H,Q,Q]
        xb = xc * bc[..., None]
        yc = (G * Lm) @ xb                                 # intra-chunk
        yc = yc + torch.exp(s)[..., None] * (Cc @ h.transpose(-1, -2))   # carried state
        yc = yc + D.view(H, P)[None, :, None, :] * xc
        y[:, c0:c1] = yc.permute(0, 2, 1, 3)
        w = torch.exp(s[..., -1:] - s)                     # [Bt,H,Q]
        h = torch.exp(s[..., -1])[..., None, None] * h + (xb * w[..., None]).transpose(-1, -2) @ Bc
    y = y.reshape(Bt, L, H * P)
    return (y, h) if return_state else y


def ssd_sharded_compose(parts, A_log, dts):
    """Sequence-parallel composition check (config 4): given per-shard results
    computed from a zero initial state — ``parts[r] = (y_r, S_r)`` — and each
    shard's dt slice, return the per-shard exclusive carries
    carry_r = sum_{j<r} (prod_{j<k<r} Lambda_k) * S_j with
    Lambda_k = exp(A_h * sum(dt over shard k)).  This is the algebra of the
    reference's carry scan (``ssm_scan.py:53-65``, ``:68-98``) lifted from
    blocks to shards.
    """
    a = -torch.exp(A_log.float())
    carries = []
    carry = torch.zeros_like(parts[0][1])
    for r, (_, S) in enumerate(parts):
        carries.append(carry.clone())
        lam = torch.exp(dts[r].float().sum(1) * a)      # [Bt,H]
        carry = lam[:, :, None, None] * carry + S
    return carries


def multihead_diag(u, A_log, B, C, dt, D, bdisc="euler", dtype=torch.float32):
    """Diagonal multi-head scan with the reference's readout.

    u [Bt,L,H] with H = n_heads*head_dim; A_log [n_heads, head_dim];
    B, C [Bt,L,n_heads,head_dim]; dt [Bt,L,n_heads]; D [H].
    Abar = exp(dt*(-exp(A_log[h,p]))) (``:64-69``), bx = (dt*B)*u (``:71-82``),
    h = Abar*h + bx (``:84-85``); per head y_h = sum_p C*h + sum_p D*u, written to
    every position p of the head's slice (``:171-187``).
    """
    u, A_log, B, C, dt, D = (t.to(dtype) for t in (u, A_log, B, C, dt, D))
    Bt, L, nh, hd = B.shape
    us = u.view(Bt, L, nh, hd)
    a = -torch.exp(A_log)                                  # [nh,hd]
    h = torch.zeros(Bt, nh, hd, dtype=dtype)
    y = torch.empty(Bt, L, nh, hd, dtype=dtype)
    Dv = D.view(nh, hd)
    for t in range(L):
        dtt = dt[:, t, :, None]                            # [Bt,nh,1]
        Abar = torch.exp(dtt * a)
        coeff = _input_coeff(dtt, a, bdisc)
        h = Abar * h + (coeff * B[:, t]) * us[:, t]
        yh = (C[:, t] * h).sum(-1) + (Dv * us[:, t]).sum(-1)
        y[:, t] = yh[..., None].expand(Bt, nh, hd)
    return y.reshape(Bt, L, nh * hd), h


def ssd_slice_scan(x, dt, A_log, B, C, D, bdisc="euler"):
    """Oracle counterpart of one rank's local pass: (y, final state, log2 of the
    whole-slice decay) from a zero initial state."""
    y, S = ssd_scan_chunked(x, dt, A_log, B, C, D, chunk=64, bdisc=bdisc)
    a = -torch.exp(A_log.float())
    d = (dt.float().sum(1) * a) * 1.4426950408889634
    return y, S, d


def ssd_carry_fixup(S_all, d_all, rank, C, dt, A_log, y):
    """Oracle counterpart of the slice chaining (in place on y): carry entering
    slice `rank` from the gathered (S, d), and its exact effect
    exp(A*cumdt(t)) * sum_n C[t,n] carry[p,n] on every output of the slice."""
    if rank == 0:
        return y
    carry = torch.zeros_like(S_all[0])
    for j in range(rank):
        carry = torch.exp2(d_all[j])[..., None, None] * carry + S_all[j]
    a = -torch.exp(A_log.float())
    Bt, L, H, N = C.shape
    P = y.shape[2] // H
    cum = torch.cumsum(dt.float() * a, dim=1)                       # [Bt,L,H]
    fix = torch.einsum("blhn,bhpn->blhp", C.float(), carry) * torch.exp(cum)[..., None]
    y += fix.reshape(Bt, L, H * P).to(y.dtype)
    return y
