"""Time-aware interpolation and the fused interpolation + SSM step (test oracle only).

Restates ``fused_interp_kernel.py:29-100`` (and its bf16/fp16 twins,
``:103-257``, which do the same arithmetic in fp32) and
``fused_ssm_interp.py:40-101``.

Reference semantics kept exactly (index mode):
* neighbours are searched per (b, t, feature tile of FTILE): the previous
  neighbour is the nearest t-k (k = 1..K) whose tile holds ANY observation, the
  next one the nearest t+k (``:43-68``);
* w = clamp((tau_t - tau_prev)/(tau_next - tau_prev), 0, 1), or 0.5 when the
  denominator is <= 1e-9 (``:80-83``);
* priority (``:94-97``): both -> lerp, prev only -> v_prev, next only ->
  v_next, none -> the current value.  Observed cells are overwritten whenever a
  neighbour exists, exactly as in the reference.

Query (time) mode extends the same rule to arbitrary sorted query times q:
lo = #{tau < q}, hi = #{tau <= q}; previous candidates are obs lo-1 .. lo-K,
next candidates hi .. hi+K-1, and the "current" observation (the fallback
value) is hi-1 when hi > lo, else none (value 0).  When the queries are the
observation times themselves and the timestamps are distinct, this equals
index mode.
"""
import torch

from .discretize import zoh_discretize


def tile_flags(M, FTILE):
    """any-observed per (b, t, tile): ``tl.sum(pm) > 0.5`` (``:51-54``)."""
    Bt, T, F = M.shape
    nt = (F + FTILE - 1) // FTILE
    pad = nt * FTILE - F
    Mf = M.float()
    if pad:
        Mf = torch.nn.functional.pad(Mf, (0, pad))
    return Mf.view(Bt, T, nt, FTILE).sum(-1) > 0.5


def interp_neighbors_index(M, K=10, FTILE=128):
    """(prev, next) [Bt,T,nt] int64 (-1 = none) in index mode (``:43-68``)."""
    fl = tile_flags(M, FTILE)
    Bt, T, nt = fl.shape
    t = torch.arange(T)[None, :, None]
    prev = torch.full((Bt, T, nt), -1, dtype=torch.long)
    nxt = torch.full((Bt, T, nt), -1, dtype=torch.long)
    for k in range(K, 0, -1):        # descending k so the nearest wins last
        tk = t - k
        ok = (tk >= 0) & fl[:, tk.clamp(min=0).squeeze(-1).squeeze(0), :]
        prev = torch.where(ok, tk.expand_as(prev), prev)
        tk = t + k
        ok = (tk < T) & fl[:, tk.clamp(max=T - 1).squeeze(-1).squeeze(0), :]
        nxt = torch.where(ok, tk.expand_as(nxt), nxt)
    return prev, nxt


def interp_neighbors_time(M, tau, q, K=10, FTILE=128):
    """(prev, next, cur) [Bt,Lq,nt] int64 in query mode (module docstring)."""
    fl = tile_flags(M, FTILE)
    Bt, T, nt = fl.shape
    Lq = q.shape[1]
    lo = torch.searchsorted(tau.contiguous(), q.contiguous(), right=False)   # [Bt,Lq]
    hi = torch.searchsorted(tau.contiguous(), q.contiguous(), right=True)
    cur = torch.where(hi > lo, hi - 1, torch.full_like(hi, -1))
    prev = torch.full((Bt, Lq, nt), -1, dtype=torch.long)
    nxt = torch.full((Bt, Lq, nt), -1, dtype=torch.long)
    bidx = torch.arange(Bt)[:, None]
    for k in range(K - 1, -1, -1):
        i = lo - 1 - k
        ok = (i >= 0)[..., None] & fl[bidx, i.clamp(min=0)]
        prev = torch.where(ok, i[..., None].expand_as(prev), prev)
        i = hi + k
        ok = (i < T)[..., None] & fl[bidx, i.clamp(max=T - 1)]
        nxt = torch.where(ok, i[..., None].expand_as(nxt), nxt)
    return prev, nxt, cur[..., None].expand(Bt, Lq, nt)


def interp_gather(V, tau, tq, prev, nxt, cur, FTILE=128):
    """Weights and priority selection (``:70-97``), fp32 math.

    V [Bt,T,F]; tau [Bt,T]; tq [Bt,Lq] query times; prev/nxt/cur [Bt,Lq,nt].
    Returns vhat [Bt,Lq,F] in fp32.
    """
    Bt, T, F = V.shape
    Vf = V.float()
    tau = tau.float()
    tq = tq.float()
    feat_tile = torch.arange(F) // FTILE
    bidx = torch.arange(Bt)[:, None, None]

    def g_tau(idx):
        return torch.where(idx >= 0, tau[bidx, idx.clamp(min=0)], torch.zeros(()))

    def g_val(idx):
        i = idx[..., feat_tile]                                   # [Bt,Lq,F]
        v = Vf[bidx, i.clamp(min=0), torch.arange(F)]
        return torch.where(i >= 0, v, torch.zeros(()))

    have_both = (prev >= 0) & (nxt >= 0)
    have_prev = (prev >= 0) & ~have_both
    have_next = (nxt >= 0) & ~have_both & ~have_prev
    tp = g_tau(prev)
    tn = g_tau(nxt)
    denom = tn - tp
    w = torch.where(denom > 1e-9, (tq[..., None] - tp) / torch.where(denom > 1e-9, denom, torch.ones(())),
                    torch.full((), 0.5))
    w = w.clamp(0.0, 1.0)
    vp = g_val(prev)
    vn = g_val(nxt)
    wf = w[..., feat_tile]
    interp = (1.0 - wf) * vp + wf * vn
    vhat = g_val(cur)
    vhat = torch.where(have_both[..., feat_tile], interp, vhat)
    vhat = torch.where(have_prev[..., feat_tile], vp, vhat)
    vhat = torch.where(have_next[..., feat_tile], vn, vhat)
    return vhat


def time_aware_interp(V, M, tau, K=10, FTILE=128):
    """``fused_time_aware_interp_kernel`` (``fused_interp_kernel.py:9-100``).
    Returns Vhat [Bt,T,F] in V's dtype (fp32 math, cast on store as in the
    bf16/fp16 kernels ``:178-181``, ``:254-257``)."""
    Bt, T, F = V.shape
    prev, nxt = interp_neighbors_index(M, K, FTILE)
    cur = torch.arange(T)[None, :, None].expand_as(prev)
    vhat = interp_gather(V, tau, tau, prev, nxt, cur, FTILE)
    return vhat.to(V.dtype)


def linspace_queries(tau, Lq):
    """Regular query grid per batch row spanning [tau[:,0], tau[:,-1]] with both
    end points exact: q_i = tau_0 + i*(tau_last - tau_0)/(Lq-1)."""
    t0 = tau[:, :1].float()
    t1 = tau[:, -1:].float()
    step = (t1 - t0) / (Lq - 1)
    q = t0 + torch.arange(Lq, dtype=torch.float32)[None, :] * step
    q[:, -1:] = t1
    return q


def interp_ssm_step(V, M, tau, Abar, Bbar, h_in, t_cur, K=10, FTILE=128):
    """``fused_interp_ssm_step_kernel`` (``fused_ssm_interp.py:11-101``):
    interpolate column t_cur then h_out = Abar*h_in + Bbar*vhat (``:95-101``).
    Returns (vhat_t [Bt,F], h_out [Bt,F])."""
    prev, nxt = interp_neighbors_index(M, K, FTILE)
    T = V.shape[1]
    cur = torch.arange(T)[None, :, None].expand_as(prev)
    vhat = interp_gather(V, tau, tau, prev, nxt, cur, FTILE)[:, t_cur]
    h_out = Abar.float() * h_in.float() + Bbar.float() * vhat
    return vhat, h_out


def interp_ssm(V, M, tau, A_log, B, C, dt, q=None, D=None, h0=None, K=10, FTILE=128,
               return_vhat=False):
    """Interpolation onto queries feeding an N-state diagonal scan (config 3).

    V [Bt,T,Dd]; M [Bt,T,Dd] (nonzero = observed); tau [Bt,T]; A_log, B, C [Dd,N];
    dt [Bt] — one step per batch row (the regular query spacing); q [Bt,Lq]
    query times, or None for index mode (queries = observation indices).
    Per (b,d,n): Abar, Bbar = ZOH(dt_b, a[d,n]) * B[d,n] (``discretize_kernel.py:38-54``),
    h = Abar*h + Bbar*vhat_q (``fused_ssm_interp.py:100``),
    y[b,q,d] = sum_n C[d,n]*h[d,n] (+ D[d]*vhat).  Returns (y, h_last[, vhat]).
    """
    Bt, T, Dd = V.shape
    N = A_log.shape[1]
    if q is None:
        prev, nxt = interp_neighbors_index(M, K, FTILE)
        cur = torch.arange(T)[None, :, None].expand_as(prev)
        tq = tau
    else:
        prev, nxt, cur = interp_neighbors_time(M, tau, q, K, FTILE)
        tq = q
    vhat = interp_gather(V, tau, tq, prev, nxt, cur, FTILE)       # [Bt,Lq,Dd]
    Lq = vhat.shape[1]
    Ab, Bb = zoh_discretize(A_log.reshape(-1), B.reshape(1, 1, -1).expand(Bt, 1, Dd * N).float(),
                            dt.float().reshape(Bt, 1))
    Ab = Ab.view(Bt, Dd, N)
    Bb = Bb.view(Bt, Dd, N)
    Cf = C.float()
    h = torch.zeros(Bt, Dd, N) if h0 is None else h0.float().clone()
    y = torch.empty(Bt, Lq, Dd)
    for t in range(Lq):
        h = Ab * h + Bb * vhat[:, t, :, None]
        yt = (Cf * h).sum(-1)
        if D is not None:
            yt = yt + D.float() * vhat[:, t]
        y[:, t] = yt
    if return_vhat:
        return y, h, vhat
    return y, h
