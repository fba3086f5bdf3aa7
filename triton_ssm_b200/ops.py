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
           "streaming_step", "multihead_ssm", "check_device_status"]


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


def ssm_forward(u, A, B, C, D, BLK=256, store_h=True):
    """Diagonal selective scan (``ssm_scan.py:239-264``).

    u, A, B, C [Bt,L,H]; D [H]; f32 or bf16 (all the same dtype).
    Returns (y, h) [Bt,L,H] (h is None when ``store_h`` is False).  ``BLK``
    is accepted for signature compatibility; the single-pass kernel has no
    block-size dependence.
    """
    del BLK
    _cuda(u, A, B, C, D)
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
    call("tssm_ssm_forward", ptr(u), ptr(A), ptr(B), ptr(C), ptr(D), ptr(y), ptr(h), Bt, L, H,
         dtype_code(u), stream_of(u))
    return y, h


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


def multihead_ssm(u, A_log, B, C, dt, D, BLK_L=256, mode="ssd", bdisc="euler", h0=None,
                  return_state=False, y=None):
    """Multi-head chunked scan (``multihead_ssm_kernel.py:19-187``).

    mode="ssd": outer-product state h[b,h,p,n] on tcgen05 tensor cores.
      u [Bt,L,H*P] bf16; A_log [H] f32 (log(-A_h)); B, C [Bt,L,H,N] bf16;
      dt [Bt,L,H] f32; D [H*P] f32; h0 [Bt,H,P,N] f32 or None.
      Returns y [Bt,L,H*P] bf16, or (y, h_last [Bt,H,P,N] f32) when
      ``return_state``.  P = 64, N in {64, 128}.
    ``BLK_L`` is accepted for signature compatibility (the kernel's chunk is
    64 tokens; results do not depend on it beyond rounding).
    """
    del BLK_L
    if mode != "ssd":
        raise ValueError("multihead_ssm: mode %r is not available" % (mode,))
    if bdisc not in _BDISC:
        raise ValueError("multihead_ssm: bdisc must be 'euler' or 'zoh'")
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
    hl = torch.empty(Bt, H, P, N, device=u.device, dtype=torch.float32) if return_state else None
    call("tssm_multihead_ssd", ptr(u), ptr(dt), ptr(A_log), ptr(B), ptr(C), ptr(D), ptr(y), ptr(h0),
         ptr(hl), Bt, L, H, P, N, _BDISC[bdisc], stream_of(u))
    return (y, hl) if return_state else y


def check_device_status(device=None):
    """Synchronise the current stream and raise ``TimeoutError`` if a kernel's
    bounded device-side wait gave up since the last check."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    s = torch.cuda.current_stream(dev)
    import ctypes
    call("tssm_check_device_status", ctypes.c_void_p(s.cuda_stream))
