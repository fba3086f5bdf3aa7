"""Mint the golden fixtures in this folder from the reference's own kernels.

Run once, in a container that holds the reference source tree:

    TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/reference

(or set TSSM_REFERENCE_DIR to that path instead of passing it).

Every fixture is produced by the reference's Triton kernels executed on the CPU
under the Triton interpreter (``TRITON_INTERPRET=1``) at tiny shapes, and saved
as ``<case>.npz`` (inputs and outputs, float32 / uint8 / int32).  Nothing at
test time imports the reference: the tests read only the ``.npz`` files.

Where the reference has no single kernel for a semantic this build needs
(the outer-product multi-head state, the per-stream streaming step, the
N-state interpolated scan), the case composes reference kernels — the ZOH
discretize kernel, ``ssm_forward`` and the streaming / fused-step kernels —
over a flattened channel axis and sums the readout over the state axis on the
host.  Each case says which reference lines it exercises.
"""
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("TSSM_REFERENCE_DIR")
if not REF or not os.path.isfile(os.path.join(REF, "ssm_scan.py")):
    sys.exit("usage: make_golden.py /path/to/reference  (the directory holding ssm_scan.py; "
             "or set TSSM_REFERENCE_DIR)")
sys.path.insert(0, REF)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import discretize_kernel as dk  # noqa: E402
import fused_interp_kernel as fik  # noqa: E402
import fused_ssm_interp as fsi  # noqa: E402
import ssm_scan  # noqa: E402
import streaming_inference_kernel as sik  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.detach().cpu().numpy()


def save(name, **arrs):
    path = os.path.join(OUT, name + ".npz")
    np.savez_compressed(path, **{k: (_np(v) if torch.is_tensor(v) else np.asarray(v))
                                 for k, v in arrs.items()})
    print("wrote", path)


def cdiv(a, b):
    return (a + b - 1) // b


# --------------------------------------------------------------------------
# reference-kernel helpers (each is one launch of a reference kernel)
# --------------------------------------------------------------------------
def ref_discretize(A_log, Bc, dt, bf16=False, BLOCK_H=32):
    """discretize_kernel.py:15-57 (fp32) / :60-94 (bf16)."""
    Bsz, T, H = Bc.shape
    Ab = torch.empty_like(Bc)
    Bb = torch.empty_like(Bc)
    kern = dk.zoh_discretize_diag_bf16_kernel if bf16 else dk.zoh_discretize_diag_kernel
    kern[(Bsz, T, cdiv(H, BLOCK_H))](A_log, Bc, dt, Ab, Bb, Bsz, T, H,
                                     *Bc.stride(), *dt.stride(), *Ab.stride(), *Bb.stride(),
                                     BLOCK_H=BLOCK_H)
    return Ab, Bb


def ref_interp(V, M, tau, K=10, FTILE=128):
    """fused_interp_kernel.py:9-100 / :103-181 / :186-257 by dtype."""
    Bsz, T, F = V.shape
    Vh = torch.empty_like(V)
    kern = {torch.float32: fik.fused_time_aware_interp_kernel,
            torch.bfloat16: fik.fused_interp_bf16_kernel,
            torch.float16: fik.fused_interp_fp16_kernel}[V.dtype]
    kern[(Bsz, T, cdiv(F, FTILE))](V, M, tau, Vh, Bsz, T, F,
                                   *V.stride(), *M.stride(), *tau.stride(), *Vh.stride(),
                                   K=K, FTILE=FTILE)
    return Vh


def ref_interp_step(V, M, tau, Abar, Bbar, h_in, Vhat, t_cur, K=10, FTILE=128):
    """fused_ssm_interp.py:11-101 (one launch = one time index)."""
    Bsz, T, F = V.shape
    h_out = torch.empty_like(h_in)
    fsi.fused_interp_ssm_step_kernel[(Bsz, cdiv(F, FTILE))](
        V, M, tau, Abar, Bbar, h_in, Vhat, h_out, Bsz, T, F,
        *V.stride(), *M.stride(), *tau.stride(), *Vhat.stride(),
        *h_in.stride(), *h_out.stride(), t_cur, K=K, FTILE=FTILE)
    return h_out


def ref_stream_inplace(vhat, h, Abar, Bbar, C, D, bf16=False, BLOCK_H=64):
    """streaming_inference_kernel.py:6-37 (fp32) / :40-71 (bf16)."""
    Bsz, H = vhat.shape
    y = torch.empty_like(vhat)
    kern = sik.streaming_ssm_inplace_bf16_kernel if bf16 else sik.streaming_ssm_inplace_kernel
    kern[(Bsz, cdiv(H, BLOCK_H))](vhat, h, Abar, Bbar, C, D, y, Bsz, H,
                                  *vhat.stride(), *h.stride(), *C.stride(), BLOCK_H=BLOCK_H)
    return y


def make_masks(g, Bsz, T, F, FTILE, p_obs, p_tile_empty):
    """Per-feature Bernoulli(p_obs) mask with whole (b, t, tile) blocks dropped."""
    m = (torch.rand(Bsz, T, F, generator=g) < p_obs)
    nt = cdiv(F, FTILE)
    drop = torch.rand(Bsz, T, nt, generator=g) < p_tile_empty
    drop = drop.repeat_interleave(FTILE, dim=2)[:, :, :F]
    return (m & ~drop).to(torch.uint8)


def main():
    g = torch.Generator().manual_seed(20261201)

    # ---- 1/2. ZOH discretize, fp32 and bf16 I/O -------------------------
    Bsz, T, H = 2, 6, 37
    neg_a = torch.exp(torch.empty(H).uniform_(np.log(0.5), np.log(16.0), generator=g))
    A_log = torch.log(neg_a)
    dt = torch.tensor([[1e-7, 5e-7, 1e-6, 6.3e-6, 1e-5, 2e-5],
                       [1e-4, 1e-3, 0.37, 1.0, 4.2, 10.0]], dtype=torch.float32)
    Bc = torch.randn(Bsz, T, H, generator=g)
    Ab, Bb = ref_discretize(A_log, Bc, dt)
    save("discretize_fp32", A_log=A_log, B=Bc, dt=dt, Abar=Ab, Bbar=Bb)
    Bc16 = Bc.bfloat16()
    Ab16, Bb16 = ref_discretize(A_log, Bc16, dt, bf16=True)
    save("discretize_bf16", A_log=A_log, B=Bc16, dt=dt, Abar=Ab16, Bbar=Bb16)

    # ---- 3/4. ssm_forward (ssm_scan.py:239-264) ----------------------------
    for name, (Bsz, L, H, BLK) in {"ssm_forward_a": (2, 300, 3, 64),
                                   "ssm_forward_b": (1, 257, 33, 256)}.items():
        u = torch.randn(Bsz, L, H, generator=g)
        A = torch.rand(Bsz, L, H, generator=g) * 0.5 + 0.5
        Bm = torch.randn(Bsz, L, H, generator=g)
        C = torch.randn(Bsz, L, H, generator=g)
        D = torch.randn(H, generator=g)
        y, h = ssm_scan.ssm_forward(u, A, Bm, C, D, BLK=BLK)
        save(name, u=u, A=A, B=Bm, C=C, D=D, BLK=BLK, y=y, h=h)

    # ---- 5. config-1 drop-in pair: discretize then ssm_forward over H'=D*N
    Bsz, L, Dd, N = 2, 50, 3, 4
    x = torch.randn(Bsz, L, Dd, generator=g)
    dt = torch.empty(Bsz, L).exponential_(1.0, generator=g).clamp_(1e-3, 10.0)
    A_log = torch.log(torch.arange(1, N + 1, dtype=torch.float32)).repeat(Dd, 1)  # [D,N]
    Bs = torch.randn(Bsz, L, N, generator=g) / np.sqrt(N)
    Cs = torch.randn(Bsz, L, N, generator=g) / np.sqrt(N)
    Dskip = torch.randn(Dd, generator=g)
    Hp = Dd * N
    B_exp = Bs[:, :, None, :].expand(Bsz, L, Dd, N).reshape(Bsz, L, Hp).contiguous()
    C_exp = Cs[:, :, None, :].expand(Bsz, L, Dd, N).reshape(Bsz, L, Hp).contiguous()
    u_exp = x[:, :, :, None].expand(Bsz, L, Dd, N).reshape(Bsz, L, Hp).contiguous()
    Ab, Bb = ref_discretize(A_log.reshape(-1).contiguous(), B_exp, dt)
    yp, hp = ssm_scan.ssm_forward(u_exp, Ab, Bb, C_exp, torch.zeros(Hp), BLK=16)
    y = yp.view(Bsz, L, Dd, N).sum(-1) + Dskip * x
    save("c1_pair", x=x, dt=dt, A_log=A_log, B=Bs, C=Cs, D=Dskip, y=y,
         h_last=hp[:, -1].reshape(Bsz, Dd, N), Abar=Ab, Bbar=Bb, y_chan=yp, h_chan=hp)

    # ---- 6. multi-head outer-product (SSD) state, Euler B (composition) ----
    Bsz, L, nh, P, N = 2, 40, 2, 4, 3
    x = torch.randn(Bsz, L, nh * P, generator=g)
    dt = torch.exp(torch.empty(Bsz, L, nh).uniform_(np.log(1e-3), 0.0, generator=g))
    A_h = -torch.exp(torch.empty(nh).uniform_(np.log(0.5), np.log(16.0), generator=g))
    A_log = torch.log(-A_h)
    Bs = torch.randn(Bsz, L, nh, N, generator=g) / np.sqrt(N)
    Cs = torch.randn(Bsz, L, nh, N, generator=g) / np.sqrt(N)
    Dskip = torch.randn(nh * P, generator=g)
    ys, hs = [], []
    for h in range(nh):
        Hp = P * N
        dummyB = torch.zeros(Bsz, L, Hp)
        Ab, _ = ref_discretize(A_log[h].repeat(Hp).contiguous(), dummyB, dt[:, :, h].contiguous())
        Bbar = (dt[:, :, h, None] * Bs[:, :, h, :])                      # Euler, [B,L,N]
        Bb_exp = Bbar[:, :, None, :].expand(Bsz, L, P, N).reshape(Bsz, L, Hp).contiguous()
        C_exp = Cs[:, :, h, None, :].expand(Bsz, L, P, N).reshape(Bsz, L, Hp).contiguous()
        u_exp = x[:, :, h * P:(h + 1) * P, None].expand(Bsz, L, P, N).reshape(Bsz, L, Hp).contiguous()
        yp, hp = ssm_scan.ssm_forward(u_exp, Ab, Bb_exp, C_exp, torch.zeros(Hp), BLK=16)
        ys.append(yp.view(Bsz, L, P, N).sum(-1))
        hs.append(hp[:, -1].view(Bsz, P, N))
    y = torch.cat(ys, dim=2) + Dskip * x
    save("ssd_composed", x=x, dt=dt, A_log=A_log, B=Bs, C=Cs, D=Dskip, y=y,
         h_last=torch.stack(hs, dim=1))

    # ---- 7. multi-head diagonal state (multihead_ssm_kernel.py semantics) --
    Bsz, L, nh, P = 2, 40, 2, 4
    x = torch.randn(Bsz, L, nh * P, generator=g)
    dt = torch.exp(torch.empty(Bsz, L, nh).uniform_(np.log(1e-3), 0.0, generator=g))
    A_log = torch.empty(nh, P).uniform_(np.log(0.5), np.log(16.0), generator=g)
    Bs = torch.randn(Bsz, L, nh, P, generator=g)
    Cs = torch.randn(Bsz, L, nh, P, generator=g)
    Dskip = torch.randn(nh * P, generator=g)
    ys = []
    for h in range(nh):
        Ab, _ = ref_discretize(A_log[h].contiguous(), torch.zeros(Bsz, L, P), dt[:, :, h].contiguous())
        Bbar = (dt[:, :, h, None] * Bs[:, :, h, :]).contiguous()
        u_h = x[:, :, h * P:(h + 1) * P].contiguous()
        yp, _ = ssm_scan.ssm_forward(u_h, Ab, Bbar, Cs[:, :, h, :].contiguous(), torch.zeros(P), BLK=16)
        yh = yp.sum(-1) + (Dskip[h * P:(h + 1) * P] * u_h).sum(-1)
        ys.append(yh[:, :, None].expand(Bsz, L, P))
    y = torch.cat(ys, dim=2)
    save("mh_diag_composed", x=x, dt=dt, A_log=A_log, B=Bs, C=Cs, D=Dskip, y=y)

    # ---- 8. time-aware interpolation, three dtypes --------------------------
    Bsz, T, F = 2, 40, 200
    V = torch.randn(Bsz, T, F, generator=g)
    M = make_masks(g, Bsz, T, F, 128, 0.7, 0.35)
    tau = torch.cumsum(torch.empty(Bsz, T).exponential_(1.0, generator=g), dim=1)
    tau[0, 10] = tau[0, 9]            # a tie: denom <= 1e-9 takes w = 0.5
    tau[1, 20:23] = tau[1, 20]
    for dtn, dty in (("fp32", torch.float32), ("bf16", torch.bfloat16), ("fp16", torch.float16)):
        Vd = V.to(dty)
        Vh = ref_interp(Vd, M, tau)
        save("interp_" + dtn, V=Vd, M=M, tau=tau, Vhat=Vh)

    # ---- 9. fused interpolation + one SSM step, all t_cur in turn ----------
    Bsz, T, F = 2, 30, 150
    V = torch.randn(Bsz, T, F, generator=g)
    M = make_masks(g, Bsz, T, F, 128, 0.7, 0.3)
    tau = torch.cumsum(torch.empty(Bsz, T).exponential_(1.0, generator=g), dim=1)
    Abar = torch.rand(F, generator=g) * 0.9 + 0.05
    Bbar = torch.randn(F, generator=g)
    h = torch.randn(Bsz, F, generator=g)
    h0 = h.clone()
    Vhat = torch.zeros(Bsz, T, F)
    hs = []
    for t in range(T):
        h = ref_interp_step(V, M, tau, Abar, Bbar, h, Vhat, t)
        hs.append(h.clone())
    save("interp_step_seq", V=V, M=M, tau=tau, Abar=Abar, Bbar=Bbar, h0=h0,
         Vhat=Vhat, h_seq=torch.stack(hs, dim=0))

    # ---- 10. interpolation onto the obs grid feeding an N-state scan -------
    Bsz, T, Dd, N = 2, 30, 150, 3
    V = torch.randn(Bsz, T, Dd, generator=g)
    M = make_masks(g, Bsz, T, Dd, 128, 0.7, 0.3)
    tau = torch.cumsum(torch.empty(Bsz, T).exponential_(1.0, generator=g), dim=1)
    A_log = torch.log(torch.arange(1, N + 1, dtype=torch.float32)).repeat(Dd, 1)
    Bp = torch.randn(Dd, N, generator=g) / np.sqrt(N)
    Cp = torch.randn(Dd, N, generator=g) / np.sqrt(N)
    dtb = torch.tensor([0.25, 0.6])
    y = torch.zeros(Bsz, T, Dd)
    h_last = torch.zeros(Bsz, Dd, N)
    Vhat_all = torch.zeros(Bsz, T, Dd)
    for b in range(Bsz):
        Ab, Bb = ref_discretize(A_log.reshape(-1).contiguous(), Bp.reshape(1, 1, -1).contiguous(),
                                dtb[b].reshape(1, 1).contiguous())
        Ab = Ab.view(Dd, N)
        Bb = Bb.view(Dd, N)
        for n in range(N):
            hb = torch.zeros(1, Dd)
            Vh = torch.zeros(1, T, Dd)
            for t in range(T):
                hb = ref_interp_step(V[b:b + 1].contiguous(), M[b:b + 1].contiguous(),
                                     tau[b:b + 1].contiguous(), Ab[:, n].contiguous(),
                                     Bb[:, n].contiguous(), hb, Vh, t)
                y[b, t] += Cp[:, n] * hb[0]
            h_last[b, :, n] = hb[0]
            Vhat_all[b] = Vh[0]
    save("interp_ssm_obsgrid", V=V, M=M, tau=tau, A_log=A_log, B=Bp, C=Cp, dt=dtb,
         y=y, h_last=h_last, Vhat=Vhat_all)

    # ---- 11. streaming in-place step, fp32 and bf16 -------------------------
    Bsz, H = 3, 70
    for dtn, bf in (("fp32", False), ("bf16", True)):
        dty = torch.bfloat16 if bf else torch.float32
        vh = torch.randn(Bsz, H, generator=g).to(dty)
        h = torch.randn(Bsz, H, generator=g).to(dty)
        Ab = (torch.rand(H, generator=g) * 0.9 + 0.05).to(dty)
        Bb = torch.randn(H, generator=g).to(dty)
        C = torch.randn(Bsz, H, generator=g).to(dty)
        D = torch.randn(H, generator=g).to(dty)
        h_in = h.clone()
        y = ref_stream_inplace(vh, h, Ab, Bb, C, D, bf16=bf)
        save("stream_inplace_" + dtn, vhat=vh, h_in=h_in, Abar=Ab, Bbar=Bb, C=C, D=D,
             h_out=h, y=y)

    # ---- 12. per-stream ZOH step with an outer-product state (composition) -
    S, H, P, N, steps = 3, 2, 4, 3, 3
    A_log = torch.empty(H).uniform_(np.log(0.5), np.log(16.0), generator=g)
    Dskip = torch.randn(H, P, generator=g)
    h = torch.randn(S, H, P, N, generator=g)
    h0 = h.clone()
    xs, dts, Bss, Css, ys = [], [], [], [], []
    for _ in range(steps):
        x = torch.randn(S, H, P, generator=g).bfloat16()
        dt = torch.empty(S).exponential_(1.0, generator=g)
        Bs = (torch.randn(S, H, N, generator=g) / np.sqrt(N)).bfloat16()
        Cs = (torch.randn(S, H, N, generator=g) / np.sqrt(N)).bfloat16()
        y = torch.zeros(S, H, P)
        for s in range(S):
            Hp = H * P * N
            A_exp = A_log[:, None, None].expand(H, P, N).reshape(Hp).contiguous()
            B_exp = Bs[s].float()[:, None, :].expand(H, P, N).reshape(1, 1, Hp).contiguous()
            Ab, Bb = ref_discretize(A_exp, B_exp, dt[s].reshape(1, 1).contiguous())
            # B_bar already carries B; unit B_bar factor into the kernel's own B_bar slot
            vh = x[s].float()[:, :, None].expand(H, P, N).reshape(1, Hp).contiguous()
            C_exp = Cs[s].float()[:, None, :].expand(H, P, N).reshape(1, Hp).contiguous()
            hs = h[s].reshape(1, Hp).contiguous()
            yp = ref_stream_inplace(vh, hs, Ab.reshape(Hp).contiguous(), Bb.reshape(Hp).contiguous(),
                                    C_exp, torch.zeros(Hp))
            h[s] = hs.view(H, P, N)
            y[s] = yp.view(H, P, N).sum(-1) + Dskip * x[s].float()
        xs.append(x); dts.append(dt); Bss.append(Bs); Css.append(Cs); ys.append(y)
    save("stream_step_composed", A_log=A_log, D=Dskip, h0=h0, x=torch.stack(xs), dt=torch.stack(dts),
         B=torch.stack(Bss), C=torch.stack(Css), y=torch.stack(ys), h_final=h)

    # ---- 13. ring-buffer ingest + forward fill + step (one H-block) --------
    Bsz, H, K = 2, 20, 4
    KR = K + 1
    ring_V = torch.zeros(Bsz, KR, H)
    ring_M = torch.zeros(Bsz, KR, H)
    ring_tau = torch.zeros(Bsz, KR)
    ring_head = torch.zeros(Bsz, dtype=torch.int32)
    h = torch.zeros(Bsz, H)
    Ab = torch.rand(H, generator=g) * 0.9 + 0.05
    Bb = torch.randn(H, generator=g)
    D = torch.randn(H, generator=g)
    init = dict(ring_V=ring_V.clone(), ring_M=ring_M.clone(), ring_tau=ring_tau.clone(),
                ring_head=ring_head.clone(), h0=h.clone())
    ev_v, ev_m, ev_t, ev_c, out_y, out_h = [], [], [], [], [], []
    tcur = torch.zeros(Bsz)
    for e in range(9):
        v_new = torch.randn(Bsz, H, generator=g)
        m_new = (torch.rand(Bsz, H, generator=g) < 0.6).float()
        if e in (2, 5):
            m_new[0].zero_()
        if e in (3, 4):
            m_new[1].zero_()
        tcur = tcur + torch.empty(Bsz).exponential_(1.0, generator=g)
        C = torch.randn(Bsz, H, generator=g)
        y = torch.empty(Bsz, H)
        sik.streaming_interp_then_ssm_kernel[(Bsz, 1)](
            ring_V, ring_M, ring_tau, ring_head, v_new, m_new, tcur.clone(), h, Ab, Bb, C, D, y,
            Bsz, H, K, *ring_V.stride(), *v_new.stride(), *h.stride(), *C.stride(),
            BLOCK_H=32, KRING=KR)
        ev_v.append(v_new); ev_m.append(m_new); ev_t.append(tcur.clone()); ev_c.append(C)
        out_y.append(y.clone()); out_h.append(h.clone())
    save("ring_stream", K=K, Abar=Ab, Bbar=Bb, D=D, v=torch.stack(ev_v), m=torch.stack(ev_m),
         tau=torch.stack(ev_t), C=torch.stack(ev_c), y=torch.stack(out_y), h=torch.stack(out_h),
         ring_V_final=ring_V, ring_M_final=ring_M, ring_tau_final=ring_tau,
         ring_head_final=ring_head, **init)

    # ---- 14. ssm_backward (ssm_scan.py:267-289) ------------------------------
    Bsz, L, H = 2, 100, 3
    u = torch.randn(Bsz, L, H, generator=g)
    A = torch.rand(Bsz, L, H, generator=g) * 0.5 + 0.5
    Bm = torch.randn(Bsz, L, H, generator=g)
    C = torch.randn(Bsz, L, H, generator=g)
    D = torch.randn(H, generator=g)
    y, h = ssm_scan.ssm_forward(u, A, Bm, C, D, BLK=32)
    dY = torch.randn(Bsz, L, H, generator=g)
    du, dA, dB, dC = ssm_scan.ssm_backward(u, A, Bm, C, h, dY, BLK=32)
    save("ssm_backward", u=u, A=A, B=Bm, C=C, D=D, h=h, dY=dY, du=du, dA=dA, dB=dB, dC=dC)

    # ---- 15. ZOH discretize backward, single H-block (no ddt race) ----------
    Bsz, T, H = 2, 4, 20
    A_log = torch.empty(H).uniform_(np.log(0.5), np.log(16.0), generator=g)
    Bc = torch.randn(Bsz, T, H, generator=g)
    dt = torch.empty(Bsz, T).exponential_(1.0, generator=g)
    Ab, Bb = ref_discretize(A_log, Bc, dt)
    dAb = torch.randn(Bsz, T, H, generator=g)
    dBb = torch.randn(Bsz, T, H, generator=g)
    dA = torch.zeros(H)
    dB = torch.empty_like(Bc)
    ddt = torch.empty_like(dt)
    dk.zoh_discretize_bwd_kernel[(Bsz, T, 1)](A_log, Bc, dt, Ab, dAb, dBb, dA, dB, ddt,
                                              Bsz, T, H, *Bc.stride(), *dt.stride(),
                                              *Ab.stride(), *dBb.stride(), BLOCK_H=32)
    save("discretize_bwd", A_log=A_log, B=Bc, dt=dt, Abar=Ab, dAbar=dAb, dBbar=dBb,
         dA_log=dA, dB=dB, ddt=ddt)


if __name__ == "__main__":
    main()
