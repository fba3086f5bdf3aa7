"""Single-step streaming updates (test oracle only).

Restates ``streaming_inference_kernel.py:6-37`` (fp32), ``:40-71`` (bf16 state)
and ``:74-156`` (ring-buffer ingest + forward fill + step).
"""
import torch

from .discretize import expm1_ref


def streaming_ssm_inplace(vhat, h, Abar, Bbar, C, D, bf16=False):
    """h_new = Abar*h + Bbar*vhat; y = C*h_new + D*vhat (``:33-37``).
    vhat, h, C [Bt,H]; Abar, Bbar, D [H] shared by all rows.  The bf16 variant
    rounds the stored state and output to bf16 (``:70-71``).
    Returns (h_new, y)."""
    f = [t.float() for t in (vhat, h, Abar, Bbar, C, D)]
    vhat, h, Abar, Bbar, C, D = f
    h_new = Abar * h + Bbar * vhat
    y = C * h_new + D * vhat
    if bf16:
        return h_new.bfloat16(), y.bfloat16()
    return h_new, y


def streaming_step(x, dt, h, A_log, B, C, D):
    """Per-stream ZOH step with an outer-product state.

    x [S,H,P]; dt [S]; h [S,H,P,N] fp32; A_log [H]; B, C [S,H,N]; D [H,P].
    a = -exp(A_log[h]); Abar = exp(dt*a); Bbar[n] = expm1_ref(dt*a)/(a+1e-12)*B[n]
    (``discretize_kernel.py:38-54``); h = Abar*h + Bbar[n]*x[p] (``:33``);
    y[p] = sum_n C[n]*h[p,n] + D[h,p]*x[p] (``:34`` plus the sum over N).
    Returns (h_new fp32, y fp32)."""
    x, dt, h, A_log, B, C, D = (t.float() for t in (x, dt, h, A_log, B, C, D))
    a = -torch.exp(A_log)                                  # [H]
    xx = dt[:, None] * a[None, :]                          # [S,H]
    Abar = torch.exp(xx)
    Bbar = (expm1_ref(xx, "fp32") / (a + 1e-12))[..., None] * B      # [S,H,N]
    h_new = Abar[..., None, None] * h + Bbar[:, :, None, :] * x[..., None]
    y = torch.einsum("shpn,shn->shp", h_new, C) + D[None] * x
    return h_new, y


def ring_interp_then_ssm(ring_V, ring_M, ring_tau, ring_head, v_new, m_new, tau_new,
                         h, Abar, Bbar, C, D, BLOCK_H=128):
    """``streaming_interp_then_ssm_kernel`` (``:74-156``) with a race-free head
    update: the new event goes to slot (head+1) % (K+1) (``:105-117``); the
    nearest older slot whose tile holds any observation is found (``:124-130``);
    the previous values are forward-filled only when the new event's tile is
    entirely missing (``:133-143``); then one step (``:146-156``).
    Tiles are BLOCK_H features wide, as the reference's H-blocks are.
    Mutates the ring tensors and h; returns y.
    """
    Bt, KR, H = ring_V.shape
    nt = (H + BLOCK_H - 1) // BLOCK_H
    y = torch.empty(Bt, H)
    for b in range(Bt):
        nh = (int(ring_head[b]) + 1) % KR
        ring_V[b, nh] = v_new[b]
        ring_M[b, nh] = m_new[b]
        ring_tau[b, nh] = tau_new[b]
        ring_head[b] = nh
        for ti in range(nt):
            sl = slice(ti * BLOCK_H, min(H, (ti + 1) * BLOCK_H))
            prev_k = -1
            for k in range(1, KR):
                rk = (nh - k + KR) % KR
                if float(ring_M[b, rk, sl].float().sum()) > 0.5:
                    prev_k = rk
                    break
            new_any = float(m_new[b, sl].float().sum()) > 0.5
            vh = v_new[b, sl].float()
            if prev_k >= 0 and not new_any:
                vh = ring_V[b, prev_k, sl].float()
            hn = Abar[sl].float() * h[b, sl].float() + Bbar[sl].float() * vh
            h[b, sl] = hn
            y[b, sl] = C[b, sl].float() * hn + D[sl].float() * vh
    return y


def mean_pool_logit(h, W, bias):
    """``mean_pool_logit_kernel`` (``streaming_inference_kernel.py:159-194``):
    out[b] = sum_{t,h} W[h] * h[b,t,h] / (T*H + 1e-9) + bias[0].

    The reference kernel does not run under the interpreter (it indexes a block
    tensor with a Python int at :190), so this restates its evident intent;
    parity for this function is pinned only by this restatement.
    """
    Bt, T, H = h.shape
    acc = (h.double() * W.double()).sum(dim=(1, 2))
    return (acc / (T * H + 1e-9) + bias.double().reshape(-1)[0]).float()
