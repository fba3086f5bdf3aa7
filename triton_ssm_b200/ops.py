"""Python operators with the reference's names and argument order.

Each wrapper validates its tensors, allocates outputs the way the reference's
host code does (``torch.empty_like`` on the input's device and dtype,
``ssm_scan.py:251-255``), and launches the sm_100a kernel on the current CUDA
stream through the C ABI.  Bad arguments raise ``ValueError``; there is no CPU
fallback.
"""
import torch

from . import _lib
from ._lib import call, dtype_code, ptr, stream_of

__all__ = ["zoh_discretize", "ssm_forward", "selective_scan", "streaming_ssm_inplace",
           "streaming_step", "multihead_ssm", "check_device_status", "fused_time_aware_interp",
           "fused_interp_ssm_step", "fused_interp_ssm", "linspace_queries", "interp_ssm_workspace_bytes",
           "ssd_carry_fixup", "ssd_carry_fixup_packed", "ssm_backward", "zoh_discretize_bwd", "streaming_interp_then_ssm",
           "dt_project_softplus", "zoh_discretize_dtproj", "mean_pool_logit"]


def _cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("tssm_b200 operators take CUDA tensors (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


def _need(t, dtypes, name):
    if t.dtype not in dtypes:
        raise ValueError("%s: dtype %s not in %s" % (name, t.dtype, dtypes))


def _lastdim(t, name):
    if t.dim() and t.stride(-1) != 1 and t.shape[-1] > 1:
        raise ValueError("%s: last dimension must be contiguous" % name)


def zoh_discretize(A_log, B, dt, out=None):
    """ZOH discretisation (``discretize_kernel.py:15-94``).

    A_log [H] f32; B [Bt,T,H] f32 or bf16; dt [Bt,T] f32.
    Returns (Abar, Bbar) [Bt,T,H] in B's dtype.
    """
    _cuda(A_log, B, dt)
    _need(B, (torch.float32, torch.bfloat16), "B")
    if B.dim() != 3 or dt.dim() != 2 or A_log.dim() != 1:
        raise ValueError("zoh_discretize: expected A_log [H], B [Bt,T,H], dt [Bt,T]")
    Bt, T, H = B.shape
    if A_log.shape[0] != H or tuple(dt.shape) != (Bt, T):
        raise ValueError("zoh_discretize: shape mismatch")
    A_log = A_log.float().contiguous()
    dt = dt.float()
    _lastdim(B, "B")
    Abar, Bbar = out if out is not None else (torch.empty_like(B), torch.empty_like(B))
    for o in (Abar, Bbar):
        if o.shape != B.shape or o.dtype != B.dtype:
            raise ValueError("zoh_discretize: out tensors must match B")
        _lastdim(o, "out")
    call("tssm_zoh_discretize", ptr(A_log), ptr(B), ptr(dt), ptr(Abar), ptr(Bbar), Bt, T, H,
         B.stride(0), B.stride(1), dt.stride(0), dt.stride(1), Abar.stride(0), Abar.stride(1),
         Bbar.stride(0), Bbar.stride(1), dtype_code(B), stream_of(B))
    return Abar, Bbar


def _dtproj_args(dt_raw, W, bias, name):
    for t, n in ((dt_raw, "dt_raw"), (W, "W"), (bias, "bias")):
        _need(t, (torch.float32,), n)
    if dt_raw.dim() != 3 or W.dim() != 2 or bias.dim() != 1:
        raise ValueError("%s: expected dt_raw [Bt,T,R], W [R,H], bias [H]" % name)
    Bt, T, R = dt_raw.shape
    if W.shape[0] != R or bias.shape[0] != W.shape[1]:
        raise ValueError("%s: shape mismatch (dt_raw %s, W %s, bias %s)" % (name, tuple(dt_raw.shape),
                                                                           tuple(W.shape), tuple(bias.shape)))
    return Bt, T, W.shape[1], R


def dt_project_softplus(dt_raw, W, bias, DT_MIN=1e-3, DT_MAX=1e-1, out=None):
    """Delta-t projection (``discretize_kernel.py:165-213``):
    dt = clamp(log(1 + exp(dt_raw @ W + bias)), DT_MIN, DT_MAX).

    dt_raw [Bt,T,R], W [R,H], bias [H], f32; R <= 256.  Returns dt [Bt,T,H].
    """
    _cuda(dt_raw, W, bias, out)
    Bt, T, H, R = _dtproj_args(dt_raw, W, bias, "dt_project_softplus")
    dt_raw, W, bias = (t.contiguous() for t in (dt_raw, W, bias))
    if out is None:
        out = torch.empty(Bt, T, H, device=dt_raw.device, dtype=torch.float32)
    elif tuple(out.shape) != (Bt, T, H) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("dt_project_softplus: out must be a contiguous f32 [Bt,T,H] tensor")
    call("tssm_dt_project_softplus", ptr(dt_raw), ptr(W), ptr(bias), ptr(out), Bt, T, H, R, float(DT_MIN),
         float(DT_MAX), stream_of(dt_raw))
    return out


def zoh_discretize_dtproj(A_log, B, dt_raw, W, bias, DT_MIN=1e-3, DT_MAX=1e-1, return_dt=False):
    """The delta-t projection fused into the ZOH discretisation, one dt per
    (b, t, h): ``dt_project_softplus`` then ``discretize_kernel.py:38-54`` with
    that dt, in one launch (dt is not written unless ``return_dt``).

    A_log [H]; B [Bt,T,H]; dt_raw [Bt,T,R]; W [R,H]; bias [H]; all f32.
    Returns (Abar, Bbar) [Bt,T,H] (and dt when ``return_dt``).
    """
    _cuda(A_log, B, dt_raw, W, bias)
    Bt, T, H, R = _dtproj_args(dt_raw, W, bias, "zoh_discretize_dtproj")
    _need(A_log, (torch.float32,), "A_log")
    _need(B, (torch.float32,), "B")
    if tuple(B.shape) != (Bt, T, H) or tuple(A_log.shape) != (H,):
        raise ValueError("zoh_discretize_dtproj: expected A_log [H] and B [Bt,T,H]")
    A_log, B, dt_raw, W, bias = (t.contiguous() for t in (A_log, B, dt_raw, W, bias))
    Abar, Bbar = torch.empty_like(B), torch.empty_like(B)
    dt = torch.empty_like(B) if return_dt else None
    call("tssm_zoh_discretize_dtproj", ptr(A_log), ptr(B), ptr(dt_raw), ptr(W), ptr(bias), ptr(Abar), ptr(Bbar),
         ptr(dt), Bt, T, H, R, float(DT_MIN), float(DT_MAX), stream_of(B))
    return (Abar, Bbar, dt) if return_dt else (Abar, Bbar)


def ssm_forward(u, A, B, C, D, BLK=256, store_h=True, pool=None):
    """Diagonal selective scan (``ssm_scan.py:239-264``).

    u, A, B, C [Bt,L,H]; D [H]; f32 or bf16 (all the same dtype).
    Returns (y, h) [Bt,L,H] (h is None when ``store_h`` is False).  ``BLK``
    is accepted for signature compatibility; the single-pass kernel has no
    block-size dependence.

    ``pool=(W, bias)`` (W [H] f32, bias [1] f32) fuses the mean-pooled logit
    head (``streaming_inference_kernel.py:159-194``) over y into the scan and
    returns (y, h, logits [Bt]).
    """
    del BLK
    _cuda(u, A, B, C, D, *(pool or ()))
    _need(u, (torch.float32, torch.bfloat16), "u")
    for t in (A, B, C, D):
        if t.dtype != u.dtype:
            raise ValueError("ssm_forward: u, A, B, C, D must share a dtype")
    if u.dim() != 3 or A.shape != u.shape or B.shape != u.shape or C.shape != u.shape \
            or D.shape != (u.shape[2],):
        raise ValueError("ssm_forward: expected u, A, B, C [Bt,L,H] and D [H]")
    u, A, B, C, D = (t.contiguous() for t in (u, A, B, C, D))
    Bt, L, H = u.shape
    y = torch.empty_like(u)
    h = torch.empty_like(u) if store_h else None
    if pool is None:
        call("tssm_ssm_forward", ptr(u), ptr(A), ptr(B), ptr(C), ptr(D), ptr(y), ptr(h), Bt, L, H,
             dtype_code(u), stream_of(u))
        return y, h
    W, bias = _pool_args(pool[0], pool[1], H, "ssm_forward")
    logits = torch.empty(Bt, device=u.device, dtype=torch.float32)
    call("tssm_ssm_forward_pool", ptr(u), ptr(A), ptr(B), ptr(C), ptr(D), ptr(y), ptr(h), ptr(W), ptr(bias),
         ptr(logits), Bt, L, H, dtype_code(u), stream_of(u))
    return y, h, logits


def _pool_args(W, bias, H, name):
    _need(W, (torch.float32,), "W")
    _need(bias, (torch.float32,), "bias")
    if tuple(W.shape) != (H,) or bias.numel() != 1:
        raise ValueError("%s: pool weight must be [H] and bias one element" % name)
    return W.contiguous(), bias.reshape(1).contiguous()


def mean_pool_logit(h, W, bias):
    """Mean-pooled logit head (``streaming_inference_kernel.py:159-194``):
    out[b] = sum_{t,h} W[h] h[b,t,h] / (T*H + 1e-9) + bias.

    h [Bt,T,H] f32 or bf16; W [H] f32; bias one element, f32.  Returns [Bt] f32.
    """
    _cuda(h, W, bias)
    _need(h, (torch.float32, torch.bfloat16), "h")
    if h.dim() != 3:
        raise ValueError("mean_pool_logit: expected h [Bt,T,H]")
    Bt, T, H = h.shape
    W, bias = _pool_args(W, bias, H, "mean_pool_logit")
    h = h.contiguous()
    out = torch.empty(Bt, device=h.device, dtype=torch.float32)
    call("tssm_mean_pool_logit", ptr(h), ptr(W), ptr(bias), ptr(out), Bt, T, H, dtype_code(h), stream_of(h))
    return out


def ssm_backward(u, A, B, C, h, dY, BLK=256):
    """Backward of the diagonal scan (``ssm_scan.py:267-289``).

    u, A, B, C, h (the forward's states), dY [Bt,L,H]; f32 or bf16 (all the
    same dtype).  Returns (du, dA, dB, dC) [Bt,L,H] with
    dH_t = C_t dY_t + A_{t+1} dH_{t+1}, du = B dH, dA = h_{t-1} dH, dB = u dH,
    dC = dY h.  As in the reference, D is a constant (no dD, no D*dY in du).
    ``BLK`` is accepted for signature compatibility.
    """
    del BLK
    _cuda(u, A, B, C, h, dY)
    _need(u, (torch.float32, torch.bfloat16), "u")
    for t in (A, B, C, h, dY):
        if t.dtype != u.dtype:
            raise ValueError("ssm_backward: u, A, B, C, h, dY must share a dtype")
        if t.shape != u.shape:
            raise ValueError("ssm_backward: expected u, A, B, C, h, dY of one shape [Bt,L,H]")
    if u.dim() != 3:
        raise ValueError("ssm_backward: expected [Bt,L,H] tensors")
    u, A, B, C, h, dY = (t.contiguous() for t in (u, A, B, C, h, dY))
    Bt, L, H = u.shape
    du, dA, dB, dC = (torch.empty_like(u) for _ in range(4))
    call("tssm_ssm_backward", ptr(u), ptr(A), ptr(B), ptr(C), ptr(h), ptr(dY), ptr(du), ptr(dA), ptr(dB),
         ptr(dC), Bt, L, H, dtype_code(u), stream_of(u))
    return du, dA, dB, dC


def zoh_discretize_bwd(A_log, B, dt, Abar, dAbar, dBbar):
    """Backward of the ZOH discretisation (``discretize_kernel.py:97-162``).

    A_log [H]; B, Abar, dAbar, dBbar [Bt,T,H]; dt [Bt,T]; f32.
    Returns (dA_log [H], dB [Bt,T,H], ddt [Bt,T]), f32.  ddt is the full sum
    over H (the reference's ddt store/atomic mix races); dA_log is a fresh
    gradient (the reference adds into a buffer its caller zeroes).
    """
    _cuda(A_log, B, dt, Abar, dAbar, dBbar)
    for t, n in ((A_log, "A_log"), (B, "B"), (dt, "dt"), (Abar, "Abar"), (dAbar, "dAbar"), (dBbar, "dBbar")):
        _need(t, (torch.float32,), n)
    if B.dim() != 3 or dt.dim() != 2 or A_log.dim() != 1:
        raise ValueError("zoh_discretize_bwd: expected A_log [H], B [Bt,T,H], dt [Bt,T]")
    Bt, T, H = B.shape
    if A_log.shape[0] != H or tuple(dt.shape) != (Bt, T) or any(t.shape != B.shape for t in (Abar, dAbar, dBbar)):
        raise ValueError("zoh_discretize_bwd: shape mismatch")
    A_log, B, dt, Abar, dAbar, dBbar = (t.contiguous() for t in (A_log, B, dt, Abar, dAbar, dBbar))
    dA_log = torch.empty_like(A_log)
    dB = torch.empty_like(B)
    ddt = torch.empty_like(dt)
    call("tssm_zoh_discretize_bwd", ptr(A_log), ptr(B), ptr(dt), ptr(Abar), ptr(dAbar), ptr(dBbar), ptr(dA_log),
         ptr(dB), ptr(ddt), Bt, T, H, stream_of(B))
    return dA_log, dB, ddt


def selective_scan(x, dt, A_log, B, C, D, return_state=True):
    """Fused ZOH discretisation + diagonal scan + readout over an N-wide state
    per channel: ``zoh_discretize`` then ``ssm_forward`` over H' = D*N with the
    readout summed over N, in one launch.

    x [Bt,L,Dm]; dt [Bt,L]; A_log [Dm,N]; B, C [Bt,L,N]; D [Dm]; all f32.
    Returns (y [Bt,L,Dm], h_last [Bt,Dm,N] or None).
    """
    _cuda(x, dt, A_log, B, C, D)
    for t, n in ((x, "x"), (dt, "dt"), (A_log, "A_log"), (B, "B"), (C, "C"), (D, "D")):
        _need(t, (torch.float32,), n)
    Bt, L, Dm = x.shape
    N = A_log.shape[1]
    if tuple(dt.shape) != (Bt, L) or tuple(A_log.shape) != (Dm, N) or \
            tuple(B.shape) != (Bt, L, N) or tuple(C.shape) != (Bt, L, N) or tuple(D.shape) != (Dm,):
        raise ValueError("selective_scan: shape mismatch")
    x, dt, A_log, B, C, D = (t.contiguous() for t in (x, dt, A_log, B, C, D))
    y = torch.empty_like(x)
    h = torch.empty(Bt, Dm, N, device=x.device, dtype=torch.float32) if return_state else None
    call("tssm_selective_scan", ptr(x), ptr(dt), ptr(A_log), ptr(B), ptr(C), ptr(D), ptr(y), ptr(h),
         Bt, L, Dm, N, stream_of(x))
    return y, h


def streaming_ssm_inplace(vhat, h, Abar, Bbar, C, D, y=None):
    """In-place streaming step with shared parameters
    (``streaming_inference_kernel.py:6-71``).  vhat, h, C [Bt,H]; Abar, Bbar,
    D [H]; f32, or bf16 (state stored back in bf16).  Mutates h; returns y."""
    _cuda(vhat, h, Abar, Bbar, C, D)
    _need(vhat, (torch.float32, torch.bfloat16), "vhat")
    for t in (h, Abar, Bbar, C, D):
        if t.dtype != vhat.dtype:
            raise ValueError("streaming_ssm_inplace: all tensors must share a dtype")
    Bt, H = vhat.shape
    if h.shape != vhat.shape or C.shape != vhat.shape or Abar.shape != (H,) or \
            Bbar.shape != (H,) or D.shape != (H,):
        raise ValueError("streaming_ssm_inplace: shape mismatch")
    for t, n in ((vhat, "vhat"), (h, "h"), (C, "C")):
        _lastdim(t, n)
    Abar, Bbar, D = (t.contiguous() for t in (Abar, Bbar, D))
    if y is None:
        y = torch.empty_strided(vhat.shape, vhat.stride(), dtype=vhat.dtype, device=vhat.device)
    call("tssm_streaming_inplace", ptr(vhat), ptr(h), ptr(Abar), ptr(Bbar), ptr(C), ptr(D), ptr(y),
         Bt, H, vhat.stride(0), h.stride(0), C.stride(0), dtype_code(vhat), stream_of(vhat))
    return y


def streaming_step(x, dt, h, A_log, B, C, D, y=None):
    """Per-stream ZOH step with an f32 outer-product state resident in HBM.

    x [S,H,P] bf16 (or f32); dt [S] f32; h [S,H,P,N] f32 (updated in place);
    A_log [H] f32; B, C [S,H,N] (x's dtype); D [H,P] f32.  Returns y [S,H,P]
    in x's dtype.
    """
    _cuda(x, dt, h, A_log, B, C, D)
    _need(x, (torch.bfloat16, torch.float32), "x")
    _need(h, (torch.float32,), "h")
    S, H, P = x.shape
    N = h.shape[-1]
    if tuple(h.shape) != (S, H, P, N) or tuple(dt.shape) != (S,) or tuple(A_log.shape) != (H,) or \
            tuple(B.shape) != (S, H, N) or tuple(C.shape) != (S, H, N) or tuple(D.shape) != (H, P):
        raise ValueError("streaming_step: shape mismatch")
    if B.dtype != x.dtype or C.dtype != x.dtype:
        raise ValueError("streaming_step: B and C must have x's dtype")
    if not h.is_contiguous():
        raise ValueError("streaming_step: the state must be contiguous (it is updated in place)")
    x, dt, A_log, B, C, D = (t.contiguous() for t in (x, dt.float(), A_log.float(), B, C, D.float()))
    if y is None:
        y = torch.empty_like(x)
    call("tssm_streaming_step", ptr(x), ptr(dt), ptr(h), ptr(A_log), ptr(B), ptr(C), ptr(D), ptr(y),
         S, H, P, N, dtype_code(x), stream_of(x))
    return y


_BDISC = {"euler": 0, "zoh": 1}


def streaming_interp_then_ssm(ring_V, ring_M, ring_tau, ring_head, v_new, m_new, tau_new, h, Abar, Bbar, C, D,
                              y=None, BLOCK_H=128):
    """Ring-buffer ingest + forward fill + one step
    (``streaming_inference_kernel.py:74-156``), race-free.

    ring_V, ring_M [Bt,K+1,H] f32, ring_tau [Bt,K+1] f32, ring_head [Bt] int32
    and h [Bt,H] f32 are updated in place; v_new, m_new, C [Bt,H]; tau_new [Bt];
    Abar, Bbar, D [H].  ``BLOCK_H`` is the feature-tile width over which mask
    sums decide "observed" (the reference's H-block; it changes results).
    Returns y [Bt,H].
    """
    _cuda(ring_V, ring_M, ring_tau, ring_head, v_new, m_new, tau_new, h, Abar, Bbar, C, D, y)
    for t, n in ((ring_V, "ring_V"), (ring_M, "ring_M"), (ring_tau, "ring_tau"), (v_new, "v_new"),
                 (m_new, "m_new"), (tau_new, "tau_new"), (h, "h"), (Abar, "Abar"), (Bbar, "Bbar"), (C, "C"),
                 (D, "D")):
        _need(t, (torch.float32,), n)
    _need(ring_head, (torch.int32,), "ring_head")
    if ring_V.dim() != 3:
        raise ValueError("streaming_interp_then_ssm: ring_V must be [Bt,K+1,H]")
    Bt, KR, H = ring_V.shape
    shapes = ((ring_M, (Bt, KR, H)), (ring_tau, (Bt, KR)), (ring_head, (Bt,)), (v_new, (Bt, H)), (m_new, (Bt, H)),
              (tau_new, (Bt,)), (h, (Bt, H)), (Abar, (H,)), (Bbar, (H,)), (C, (Bt, H)), (D, (H,)))
    for t, shp in shapes:
        if tuple(t.shape) != shp:
            raise ValueError("streaming_interp_then_ssm: expected shape %s, got %s" % (shp, tuple(t.shape)))
    for t in (ring_V, ring_M, ring_tau, ring_head, h):
        if not t.is_contiguous():
            raise ValueError("streaming_interp_then_ssm: ring tensors and h are updated in place and must be "
                             "contiguous")
    v_new, m_new, tau_new, Abar, Bbar, C, D = (t.contiguous() for t in (v_new, m_new, tau_new, Abar, Bbar, C, D))
    if y is None:
        y = torch.empty_like(v_new)
    elif tuple(y.shape) != (Bt, H) or y.dtype != torch.float32 or not y.is_contiguous():
        raise ValueError("streaming_interp_then_ssm: y must be a contiguous f32 [Bt,H] tensor")
    call("tssm_ring_ingest_step", ptr(ring_V), ptr(ring_M), ptr(ring_tau), ptr(ring_head), ptr(v_new), ptr(m_new),
         ptr(tau_new), ptr(h), ptr(Abar), ptr(Bbar), ptr(C), ptr(D), ptr(y), Bt, H, KR - 1, int(BLOCK_H),
         stream_of(h))
    return y


def multihead_ssm(u, A_log, B, C, dt, D, BLK_L=256, mode="ssd", bdisc="euler", h0=None,
                  return_state=False, y=None, return_decay=False, pieces=1, state_out=None, decay_out=None):
    """Multi-head chunked scan (``multihead_ssm_kernel.py:19-187``).

    mode="diag": the reference's own diagonal state h[b,h,p]
      (``multihead_ssm_kernel.py:19-187``): u [Bt,L,H*P]; A_log [H,P];
      B, C [Bt,L,H,P]; dt [Bt,L,H]; D [H*P]; f32 or bf16 (u, B, C alike).
      Returns y [Bt,L,H*P], each head's readout broadcast over its slice.
    mode="ssd": outer-product state h[b,h,p,n] on tcgen05 tensor cores.
      u [Bt,L,H*P] bf16; A_log [H] f32 (log(-A_h)); B, C [Bt,L,H,N] bf16;
      dt [Bt,L,H] f32; D [H*P] f32; h0 [Bt,H,P,N] f32 or None.
      Returns y [Bt,L,H*P] bf16, or (y, h_last [Bt,H,P,N] f32) when
      ``return_state``; with ``return_decay`` also the log2 of the
      whole-sequence decay per (b, h), [Bt,H] f32.  P = 64, N in {64, 128}.
    ``BLK_L`` is accepted for signature compatibility (the kernel's chunk is
    64 tokens; results do not depend on it beyond rounding).
    ``pieces`` (mode "ssd", no h0, L a multiple of 64*pieces): each sequence
    is scanned as that many equal pieces at once, each from a zero state, and
    the pieces are chained by ``tssm_ssd_carry_fixup_pieces`` (the bf16
    outputs of a piece's leading tokens are rounded twice).  For few long
    sequences this spreads the work over more SMs.
    ``state_out`` [Bt,H,P,N] f32 / ``decay_out`` [Bt,H] f32 (mode "ssd"):
    contiguous tensors that receive the returned state / decay (for example
    views into a collective's send buffer), so no copy follows.
    """
    del BLK_L
    if pieces != 1:
        return _multihead_ssd_pieces(u, A_log, B, C, dt, D, int(pieces), bdisc, h0, return_state, y,
                                     return_decay, state_out, decay_out)
    if bdisc not in _BDISC:
        raise ValueError("multihead_ssm: bdisc must be 'euler' or 'zoh'")
    if mode == "diag":
        if return_state or return_decay or h0 is not None:
            raise ValueError("multihead_ssm: mode 'diag' returns y only")
        return _multihead_diag(u, A_log, B, C, dt, D, bdisc, y)
    if mode != "ssd":
        raise ValueError("multihead_ssm: mode must be 'ssd' or 'diag' (got %r)" % (mode,))
    _cuda(u, A_log, B, C, dt, D, h0)
    _need(u, (torch.bfloat16,), "u")
    _need(B, (torch.bfloat16,), "B")
    _need(C, (torch.bfloat16,), "C")
    Bt, L, HP = u.shape
    if B.dim() != 4:
        raise ValueError("multihead_ssm: B must be [Bt,L,H,N]")
    H, N = B.shape[2], B.shape[3]
    if HP % H:
        raise ValueError("multihead_ssm: u's last dim must be H*P")
    P = HP // H
    if tuple(B.shape) != (Bt, L, H, N) or tuple(C.shape) != (Bt, L, H, N) or \
            tuple(dt.shape) != (Bt, L, H) or tuple(A_log.shape) != (H,) or tuple(D.shape) != (HP,):
        raise ValueError("multihead_ssm: shape mismatch")
    if h0 is not None and tuple(h0.shape) != (Bt, H, P, N):
        raise ValueError("multihead_ssm: h0 must be [Bt,H,P,N]")
    u, B, C = (t.contiguous() for t in (u, B, C))
    dt, A_log, D = (t.float().contiguous() for t in (dt, A_log, D))
    h0 = h0.float().contiguous() if h0 is not None else None
    if y is None:
        y = torch.empty_like(u)
    hl = _out_tensor(state_out, (Bt, H, P, N), u.device, "state_out") if return_state else None
    dl = _out_tensor(decay_out, (Bt, H), u.device, "decay_out") if return_decay else None
    call("tssm_multihead_ssd", ptr(u), ptr(dt), ptr(A_log), ptr(B), ptr(C), ptr(D), ptr(y), ptr(h0),
         ptr(hl), ptr(dl), Bt, L, H, P, N, _BDISC[bdisc], stream_of(u))
    out = [y]
    if return_state:
        out.append(hl)
    if return_decay:
        out.append(dl)
    return out[0] if len(out) == 1 else tuple(out)


def _out_tensor(t, shape, device, name):
    """A caller-given f32 output (checked) or a new one."""
    if t is None:
        return torch.empty(shape, device=device, dtype=torch.float32)
    if tuple(t.shape) != tuple(shape) or t.dtype != torch.float32 or not t.is_contiguous() or t.device != device:
        raise ValueError("%s must be a contiguous f32 tensor of shape %s on %s" % (name, tuple(shape), device))
    return t


def _multihead_ssd_pieces(u, A_log, B, C, dt, D, K, bdisc, h0, return_state, y, return_decay, state_out=None,
                          decay_out=None):
    if K < 1 or h0 is not None:
        raise ValueError("multihead_ssm: pieces must be >= 1 and h0 None when pieces > 1")
    _cuda(u, A_log, B, C, dt, D)
    Bt, L, HP = u.shape
    if B.dim() != 4 or L % (64 * K):
        raise ValueError("multihead_ssm: L must be a multiple of 64*pieces")
    H, N = B.shape[2], B.shape[3]
    P = HP // H
    u, B, C = (t.contiguous() for t in (u, B, C))
    dt = dt.float().contiguous()
    A_log = A_log.float().contiguous()
    if y is None:
        y = torch.empty_like(u)
    Lp = L // K
    _, S, d = multihead_ssm(u.view(Bt * K, Lp, HP), A_log, B.view(Bt * K, Lp, H, N), C.view(Bt * K, Lp, H, N),
                            dt.view(Bt * K, Lp, H), D, bdisc=bdisc, y=y.view(Bt * K, Lp, HP),
                            return_state=True, return_decay=True)
    call("tssm_ssd_carry_fixup_pieces", ptr(S), ptr(d), K, ptr(C), ptr(dt), ptr(A_log), ptr(y), Bt, L, H, P,
         N, stream_of(y))
    out = [y]
    hl = _out_tensor(state_out, (Bt, H, P, N), u.device, "state_out") if return_state else None
    dl = _out_tensor(decay_out, (Bt, H), u.device, "decay_out") if return_decay else None
    if return_state or return_decay:   # the pieces chained in order, as the fix-up chains them
        call("tssm_ssd_pieces_final_state", ptr(S), ptr(d), K, ptr(hl), ptr(dl), Bt, H, P, N, stream_of(y))
    if return_state:
        out.append(hl)
    if return_decay:
        out.append(dl)
    return out[0] if len(out) == 1 else tuple(out)


def ssd_carry_fixup(S_all, decay_log2_all, rank, C, dt, A_log, y):
    """Chain a sequence slice to the slices before it (in place on ``y``).

    S_all [R,Bt,H,P,N] f32 and decay_log2_all [R,Bt,H] f32 are every rank's
    final state and whole-slice log2 decay from ``multihead_ssm(...,
    return_state=True, return_decay=True)``; C [Bt,L,H,N] bf16, dt [Bt,L,H]
    f32 and y [Bt,L,H*P] bf16 are this rank's slice.  See
    ``tssm_ssd_carry_fixup`` in include/tssm.h.
    """
    _cuda(S_all, decay_log2_all, C, dt, A_log, y)
    R, Bt, H, P, N = S_all.shape
    L = C.shape[1]
    if tuple(decay_log2_all.shape) != (R, Bt, H) or tuple(C.shape) != (Bt, L, H, N) or \
            tuple(dt.shape) != (Bt, L, H) or tuple(y.shape) != (Bt, L, H * P):
        raise ValueError("ssd_carry_fixup: shape mismatch")
    if not (S_all.is_contiguous() and decay_log2_all.is_contiguous() and C.is_contiguous() and
            dt.is_contiguous() and y.is_contiguous()):
        raise ValueError("ssd_carry_fixup: tensors must be contiguous")
    call("tssm_ssd_carry_fixup", ptr(S_all), ptr(decay_log2_all), int(rank), R, ptr(C), ptr(dt),
         ptr(A_log.float().contiguous()), ptr(y), Bt, L, H, P, N, stream_of(y))
    return y


def ssd_carry_fixup_packed(packed, rank, C, dt, A_log, y, P=64):
    """``ssd_carry_fixup`` reading the slices' carries from one packed buffer
    [R, Bt*H*P*N + Bt*H] f32, as one all-gather of every rank's
    [final state | log2 decay] lays them out (``tssm_ssd_carry_fixup_packed``).
    C [Bt,L,H,N] bf16, dt [Bt,L,H] f32 and y [Bt,L,H*P] bf16 are this rank's
    slice; y is fixed in place."""
    _cuda(packed, C, dt, A_log, y)
    Bt, L, H, N = C.shape
    R = packed.shape[0]
    if packed.dim() != 2 or packed.shape[1] != Bt * H * P * N + Bt * H or packed.dtype != torch.float32 or \
            tuple(dt.shape) != (Bt, L, H) or tuple(y.shape) != (Bt, L, H * P):
        raise ValueError("ssd_carry_fixup_packed: shape mismatch")
    if not (packed.is_contiguous() and C.is_contiguous() and dt.is_contiguous() and y.is_contiguous()):
        raise ValueError("ssd_carry_fixup_packed: tensors must be contiguous")
    call("tssm_ssd_carry_fixup_packed", ptr(packed), int(rank), R, ptr(C), ptr(dt),
         ptr(A_log.float().contiguous()), ptr(y), Bt, L, H, P, N, stream_of(y))
    return y


def check_device_status(device=None):
    """Synchronise the current stream and raise ``TimeoutError`` if a kernel's
    bounded device-side wait gave up since the last check."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    s = torch.cuda.current_stream(dev)
    import ctypes
    call("tssm_check_device_status", ctypes.c_void_p(s.cuda_stream))


def _mask_code(M):
    if M.dtype in (torch.uint8, torch.bool):
        return _lib.U8
    if M.dtype == torch.float32:
        return _lib.F32
    raise ValueError("mask dtype must be uint8, bool or float32 (got %s)" % M.dtype)


def _mask(M):
    return M.view(torch.uint8) if M.dtype == torch.bool else M


def fused_time_aware_interp(V, M, tau, K=10, FTILE=128, out=None):
    """Time-aware interpolation (``fused_interp_kernel.py:9-257``).

    V [Bt,T,F] f32/bf16/f16; M [Bt,T,F] uint8/bool/f32 (observed where > 0.5);
    tau [Bt,T] f32.  Returns Vhat in V's dtype.
    """
    _cuda(V, M, tau)
    _need(V, (torch.float32, torch.bfloat16, torch.float16), "V")
    if V.dim() != 3 or M.shape != V.shape or tuple(tau.shape) != tuple(V.shape[:2]):
        raise ValueError("fused_time_aware_interp: expected V, M [Bt,T,F] and tau [Bt,T]")
    M = _mask(M)
    tau = tau.float()
    for t, n in ((V, "V"), (M, "M"), (tau, "tau")):
        _lastdim(t, n)
    out = torch.empty_like(V) if out is None else out
    Bt, T, F = V.shape
    call("tssm_time_aware_interp", ptr(V), ptr(M), ptr(tau), ptr(out), Bt, T, F, V.stride(0), V.stride(1),
         M.stride(0), M.stride(1), tau.stride(0), out.stride(0), out.stride(1), int(K), int(FTILE),
         dtype_code(V), _mask_code(M), stream_of(V))
    return out


def fused_interp_ssm_step(V, M, tau, A_bar, B_bar, h_in, Vhat=None, h_out=None, t_cur=0, K=10, FTILE=128):
    """Interpolation at ``t_cur`` fused with one SSM step
    (``fused_ssm_interp.py:11-101``): writes Vhat[:, t_cur] (when given) and
    returns h_out = A_bar*h_in + B_bar*vhat.  All f32 except the mask."""
    _cuda(V, M, tau, A_bar, B_bar, h_in, Vhat, h_out)
    for t, n in ((V, "V"), (tau, "tau"), (A_bar, "A_bar"), (B_bar, "B_bar"), (h_in, "h_in")):
        _need(t, (torch.float32,), n)
    Bt, T, F = V.shape
    if M.shape != V.shape or tuple(h_in.shape) != (Bt, F) or tuple(A_bar.shape) != (F,) or \
            tuple(B_bar.shape) != (F,):
        raise ValueError("fused_interp_ssm_step: shape mismatch")
    M = _mask(M)
    A_bar, B_bar = A_bar.contiguous(), B_bar.contiguous()
    h_out = torch.empty_like(h_in) if h_out is None else h_out
    so = (Vhat.stride(0), Vhat.stride(1)) if Vhat is not None else (0, 0)
    call("tssm_interp_ssm_step", ptr(V), ptr(M), ptr(tau), ptr(A_bar), ptr(B_bar), ptr(h_in), ptr(Vhat),
         ptr(h_out), Bt, T, F, V.stride(0), V.stride(1), M.stride(0), M.stride(1), tau.stride(0), so[0], so[1],
         h_in.stride(0), h_out.stride(0), int(t_cur), int(K), int(FTILE), _mask_code(M), stream_of(V))
    return h_out


def linspace_queries(tau, L_q):
    """Regular query grid per batch row over [tau[:,0], tau[:,-1]], end points exact."""
    t0 = tau[:, :1].float()
    t1 = tau[:, -1:].float()
    step = (t1 - t0) / max(1, L_q - 1)
    q = t0 + torch.arange(L_q, device=tau.device, dtype=torch.float32)[None, :] * step
    q[:, -1:] = t1
    return q.contiguous()


def interp_ssm_workspace_bytes(Bt, T, D, L_q, FTILE=128):
    _lib.load_library()
    return int(_lib.load_library().tssm_interp_ssm_workspace_size(Bt, T, D, L_q, FTILE))


def fused_interp_ssm(V, M, tau, A_log, B, C, L_q=None, q=None, dt=None, D=None, K=10, FTILE=128,
                     return_state=False, return_vhat=False, workspace=None, static_scratch=False):
    """Interpolation of irregular observations onto query times fused with an
    N-state diagonal scan (config 3): the composition of
    ``fused_time_aware_interp_kernel`` and the step of
    ``fused_interp_ssm_step_kernel`` at every query, in one pass.

    V [Bt,T,D] f32; M [Bt,T,D] uint8/bool/f32; tau [Bt,T] f32 (sorted);
    A_log, B, C [D,N] f32; D [D] f32 or None.
    Queries: ``q`` [Bt,L_q] sorted times; or ``L_q`` for a regular grid over
    each row's [tau_0, tau_last]; or neither for index mode (the queries are the
    observations, the reference's own semantics).
    dt [Bt] f32: discretisation step per row; defaults to the regular query spacing.
    Returns y [Bt,L_q,D] f32 (+ h_last [Bt,D,N], + vhat [Bt,L_q,D]).
    ``static_scratch``: take the scratch from the library's fixed 8 MiB array
    (``tssm_interp_ssm_static_scratch``) instead of a workspace tensor, for
    callers that must not allocate device scratch per call; the outputs are
    still allocated here.  Calls that overlap on the GPU share that array.
    """
    _cuda(V, M, tau, A_log, B, C, q, dt, D)
    _need(V, (torch.float32,), "V")
    Bt, T, Dm = V.shape
    N = A_log.shape[-1]
    if M.shape != V.shape or tuple(tau.shape) != (Bt, T) or tuple(A_log.shape) != (Dm, N) or \
            tuple(B.shape) != (Dm, N) or tuple(C.shape) != (Dm, N) or (D is not None and tuple(D.shape) != (Dm,)):
        raise ValueError("fused_interp_ssm: shape mismatch")
    if q is None and L_q is not None:
        q = linspace_queries(tau, int(L_q))
    if q is not None:
        q = q.float().contiguous()
        if q.dim() != 2 or q.shape[0] != Bt:
            raise ValueError("fused_interp_ssm: q must be [Bt,L_q]")
        Lq = q.shape[1]
    else:
        Lq = T
    if dt is None:
        if q is None:
            raise ValueError("fused_interp_ssm: index mode needs an explicit dt [Bt]")
        dt = ((tau[:, -1] - tau[:, 0]).float() / max(1, Lq - 1)).contiguous()
    if tuple(dt.shape) != (Bt,):
        raise ValueError("fused_interp_ssm: dt must be [Bt]")
    M = _mask(M).contiguous()
    V, tau = V.contiguous(), tau.float().contiguous()
    A_log, B, C = (t.float().contiguous() for t in (A_log, B, C))
    D = D.float().contiguous() if D is not None else None
    dt = dt.float().contiguous()
    need = int(_lib.load_library().tssm_interp_ssm_workspace_size(Bt, T, Dm, Lq, int(FTILE)))
    if need < 0:
        raise ValueError("fused_interp_ssm: sizes out of range")
    y = torch.empty(Bt, Lq, Dm, device=V.device, dtype=torch.float32)
    hl = torch.empty(Bt, Dm, N, device=V.device, dtype=torch.float32) if return_state else None
    vh = torch.empty(Bt, Lq, Dm, device=V.device, dtype=torch.float32) if return_vhat else None
    if static_scratch:
        call("tssm_interp_ssm_static_scratch", ptr(V), ptr(M), ptr(tau), ptr(q), ptr(A_log), ptr(B), ptr(C),
             ptr(D), ptr(dt), ptr(y), ptr(hl), ptr(vh), Bt, T, Dm, N, Lq, int(K), int(FTILE), _mask_code(M),
             stream_of(V))
    else:
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=V.device)
        call("tssm_interp_ssm", ptr(V), ptr(M), ptr(tau), ptr(q), ptr(A_log), ptr(B), ptr(C), ptr(D), ptr(dt),
             ptr(y), ptr(hl), ptr(vh), ptr(workspace), workspace.numel(), Bt, T, Dm, N, Lq, int(K), int(FTILE),
             _mask_code(M), stream_of(V))
    out = [y]
    if return_state:
        out.append(hl)
    if return_vhat:
        out.append(vh)
    return out[0] if len(out) == 1 else tuple(out)


def _multihead_diag(u, A_log, B, C, dt, D, bdisc, y):
    _cuda(u, A_log, B, C, dt, D, y)
    _need(u, (torch.float32, torch.bfloat16), "u")
    if B.dtype != u.dtype or C.dtype != u.dtype:
        raise ValueError("multihead_ssm(diag): u, B, C must share a dtype")
    Bt, L, HP = u.shape
    nh, hd = A_log.shape
    if nh * hd != HP or tuple(B.shape) != (Bt, L, nh, hd) or tuple(C.shape) != (Bt, L, nh, hd) or \
            tuple(dt.shape) != (Bt, L, nh) or tuple(D.shape) != (HP,):
        raise ValueError("multihead_ssm(diag): shape mismatch")
    u, B, C = (t.contiguous() for t in (u, B, C))
    A_log, dt, D = (t.float().contiguous() for t in (A_log, dt, D))
    y = torch.empty_like(u) if y is None else y
    call("tssm_multihead_diag", ptr(u), ptr(A_log), ptr(B), ptr(C), ptr(dt), ptr(D), ptr(y), Bt, L, nh, hd,
         _BDISC[bdisc], dtype_code(u), stream_of(u))
    return y
