"""Drop-in shims for the reference's raw kernel calls.

The reference's host code launches kernels as ``kernel[grid](*args, **constexprs)``
with the argument lists of its Triton kernels.  The objects here accept exactly
those calls (same positional arguments, same meaning) and run the sm_100a
kernels through the C ABI instead; the grid and the tiling constexprs
(BLOCK_H, ...) are accepted and ignored, because the CUDA kernels choose their
own launch.  Namespaces are named after the reference modules:

    from triton_ssm_b200.compat import discretize_kernel as dk
    dk.zoh_discretize_diag_kernel[(B, T, nblk)](A_log, Bc, dt, Abar, Bbar, B, T, H, *strides, BLOCK_H=32)
"""
import types

import torch

from . import ops
from ._lib import call, dtype_code, ptr, stream_of, F32, BF16


class _Launchable:
    """``obj[grid](*args, **kw)`` -> ``fn(*args, **kw)`` (the grid is not needed)."""

    def __init__(self, name, fn):
        self.__name__ = name
        self._fn = fn

    def __getitem__(self, grid):
        return self._fn

    def __call__(self, *a, **k):
        raise TypeError("%s is launched as %s[grid](...)" % (self.__name__, self.__name__))


def _f32(t):
    return t if t.dtype == torch.float32 else t.float()


# ------------------------------------------------------------- discretize_kernel.py
def _zoh(io_dtype):
    def run(A_ptr, B_ptr, dt_ptr, Abar_ptr, Bbar_ptr, B, T, H, stride_Bb, stride_Bt, stride_Bh,
            stride_db, stride_dt, stride_ab, stride_at, stride_ah, stride_bb, stride_bt, stride_bh,
            BLOCK_H=None, **_):
        ops._cuda(A_ptr, B_ptr, dt_ptr, Abar_ptr, Bbar_ptr)
        if B_ptr.dtype != io_dtype or Abar_ptr.dtype != io_dtype or Bbar_ptr.dtype != io_dtype:
            raise ValueError("expected %s B, Abar, Bbar" % io_dtype)
        if (stride_Bh, stride_ah, stride_bh) != (1, 1, 1):
            raise ValueError("the H dimension must be contiguous (as the reference assumes)")
        A = _f32(A_ptr).contiguous()
        dt = _f32(dt_ptr)
        call("tssm_zoh_discretize", ptr(A), ptr(B_ptr), ptr(dt), ptr(Abar_ptr), ptr(Bbar_ptr), int(B), int(T), int(H),
             int(stride_Bb), int(stride_Bt), int(dt.stride(0) if dt is not dt_ptr else stride_db),
             int(dt.stride(1) if dt is not dt_ptr else stride_dt), int(stride_ab), int(stride_at), int(stride_bb),
             int(stride_bt), F32 if io_dtype == torch.float32 else BF16, stream_of(B_ptr))
    return run


def _not_built(name, instead):
    def run(*a, **k):
        raise NotImplementedError("%s is not part of this build; use %s" % (name, instead))
    return run


discretize_kernel = types.SimpleNamespace(
    zoh_discretize_diag_kernel=_Launchable("zoh_discretize_diag_kernel", _zoh(torch.float32)),
    zoh_discretize_diag_bf16_kernel=_Launchable("zoh_discretize_diag_bf16_kernel", _zoh(torch.bfloat16)),
    zoh_discretize_bwd_kernel=_Launchable("zoh_discretize_bwd_kernel",
                                          _not_built("zoh_discretize_bwd_kernel", "the forward ops (backward is next)")),
    dt_project_softplus_kernel=_Launchable("dt_project_softplus_kernel",
                                           _not_built("dt_project_softplus_kernel", "torch ops for the projection")),
)


# ------------------------------------------------------------- ssm_scan.py
def _ssm_backward(*a, **k):
    raise NotImplementedError("ssm_backward is not part of this build yet")


ssm_scan = types.SimpleNamespace(ssm_forward=ops.ssm_forward, ssm_backward=_ssm_backward)


# ------------------------------------------------------------- fused_interp_kernel.py
def _interp(v_dtype):
    def run(V_ptr, M_ptr, tau_ptr, Vhat_ptr, B, T, F, stride_vb, stride_vt, stride_vf, stride_mb, stride_mt,
            stride_mf, stride_tb, stride_tt, stride_ob, stride_ot, stride_of, K=10, FTILE=128, **_):
        ops._cuda(V_ptr, M_ptr, tau_ptr, Vhat_ptr)
        if V_ptr.dtype != v_dtype or Vhat_ptr.dtype != v_dtype:
            raise ValueError("expected %s V and Vhat" % v_dtype)
        if (stride_vf, stride_mf, stride_of, stride_tt) != (1, 1, 1, 1):
            raise ValueError("the feature and time dimensions of tau must be contiguous")
        M = ops._mask(M_ptr)
        tau = _f32(tau_ptr)
        call("tssm_time_aware_interp", ptr(V_ptr), ptr(M), ptr(tau), ptr(Vhat_ptr), int(B), int(T), int(F),
             int(stride_vb), int(stride_vt), int(stride_mb), int(stride_mt), int(tau.stride(0)), int(stride_ob),
             int(stride_ot), int(K), int(FTILE), dtype_code(V_ptr), ops._mask_code(M), stream_of(V_ptr))
    return run


fused_interp_kernel = types.SimpleNamespace(
    fused_time_aware_interp_kernel=_Launchable("fused_time_aware_interp_kernel", _interp(torch.float32)),
    fused_interp_bf16_kernel=_Launchable("fused_interp_bf16_kernel", _interp(torch.bfloat16)),
    fused_interp_fp16_kernel=_Launchable("fused_interp_fp16_kernel", _interp(torch.float16)),
)


# ------------------------------------------------------------- fused_ssm_interp.py
def _interp_step(V_ptr, M_ptr, tau_ptr, A_bar_ptr, B_bar_ptr, h_in_ptr, Vhat_ptr, h_out_ptr, B, T, F,
                 stride_vb, stride_vt, stride_vf, stride_mb, stride_mt, stride_mf, stride_tb, stride_tt,
                 stride_ob, stride_ot, stride_of, stride_hib, stride_hif, stride_hob, stride_hof, t_cur,
                 K=10, FTILE=128, **_):
    ops._cuda(V_ptr, M_ptr, tau_ptr, A_bar_ptr, B_bar_ptr, h_in_ptr, Vhat_ptr, h_out_ptr)
    M = ops._mask(M_ptr)
    call("tssm_interp_ssm_step", ptr(V_ptr), ptr(M), ptr(tau_ptr), ptr(A_bar_ptr.contiguous()),
         ptr(B_bar_ptr.contiguous()), ptr(h_in_ptr), ptr(Vhat_ptr), ptr(h_out_ptr), int(B), int(T), int(F),
         int(stride_vb), int(stride_vt), int(stride_mb), int(stride_mt), int(stride_tb), int(stride_ob),
         int(stride_ot), int(stride_hib), int(stride_hob), int(t_cur), int(K), int(FTILE), ops._mask_code(M),
         stream_of(V_ptr))


fused_ssm_interp = types.SimpleNamespace(
    fused_interp_ssm_step_kernel=_Launchable("fused_interp_ssm_step_kernel", _interp_step))


# ------------------------------------------------------------- streaming_inference_kernel.py
def _stream(dtype):
    def run(vhat_ptr, h_ptr, Abar_ptr, Bbar_ptr, C_ptr, D_ptr, y_ptr, B, H, stride_vb, stride_vh, stride_hb,
            stride_hh, stride_cb, stride_ch, BLOCK_H=None, **_):
        ops._cuda(vhat_ptr, h_ptr, Abar_ptr, Bbar_ptr, C_ptr, D_ptr, y_ptr)
        if vhat_ptr.dtype != dtype:
            raise ValueError("expected %s tensors" % dtype)
        call("tssm_streaming_inplace", ptr(vhat_ptr), ptr(h_ptr), ptr(Abar_ptr.contiguous()), ptr(Bbar_ptr.contiguous()),
             ptr(C_ptr), ptr(D_ptr.contiguous()), ptr(y_ptr), int(B), int(H), int(stride_vb), int(stride_hb),
             int(stride_cb), dtype_code(vhat_ptr), stream_of(vhat_ptr))
    return run


streaming_inference_kernel = types.SimpleNamespace(
    streaming_ssm_inplace_kernel=_Launchable("streaming_ssm_inplace_kernel", _stream(torch.float32)),
    streaming_ssm_inplace_bf16_kernel=_Launchable("streaming_ssm_inplace_bf16_kernel", _stream(torch.bfloat16)),
)

__all__ = ["discretize_kernel", "ssm_scan", "fused_interp_kernel", "fused_ssm_interp", "streaming_inference_kernel"]
