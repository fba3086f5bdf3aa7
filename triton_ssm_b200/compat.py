"""Drop-in shims for the reference's raw kernel calls.

The reference's host code launches kernels as ``kernel[grid](*args, **constexprs)``
with the argument lists of its Triton kernels.  The objects here accept exactly
those calls (same positional arguments, same meaning) and run the sm_100a
kernels through the C ABI instead; the grid and the tiling constexprs
(BLOCK_H, ...) are accepted and ignored, because the CUDA kernels choose their
own launch.  Every launched @triton.jit kernel of the six reference files has a shim here
except the model glue listed in NOT_PROVIDED.  Namespaces are named after the
reference modules:

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


def _zoh_bwd(A_ptr, B_ptr, dt_ptr, Abar_ptr, dAbar_ptr, dBbar_ptr, dA_ptr, dB_ptr, ddt_ptr, B, T, H, stride_Bb,
             stride_Bt, stride_Bh, stride_db, stride_dt, stride_ab, stride_at, stride_ah, stride_bb, stride_bt,
             stride_bh, BLOCK_H=None, **_):
    """zoh_discretize_bwd_kernel (discretize_kernel.py:97-162).  As in the
    reference, dA is accumulated into the caller's buffer (it atomically adds
    every (b, t) contribution); dB and ddt are written, ddt as the full sum over
    H (the reference's per-block store/atomic mix races when H spans blocks)."""
    ops._cuda(A_ptr, B_ptr, dt_ptr, Abar_ptr, dAbar_ptr, dBbar_ptr, dA_ptr, dB_ptr, ddt_ptr)
    for t in (B_ptr, dt_ptr, Abar_ptr, dAbar_ptr, dBbar_ptr, dA_ptr, dB_ptr, ddt_ptr):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("zoh_discretize_bwd_kernel: contiguous f32 tensors expected")
    if (int(B), int(T), int(H)) != tuple(B_ptr.shape):
        raise ValueError("zoh_discretize_bwd_kernel: B, T, H do not match the tensors")
    dA = torch.empty(int(H), device=A_ptr.device, dtype=torch.float32)
    call("tssm_zoh_discretize_bwd", ptr(_f32(A_ptr).contiguous()), ptr(B_ptr), ptr(dt_ptr), ptr(Abar_ptr),
         ptr(dAbar_ptr), ptr(dBbar_ptr), ptr(dA), ptr(dB_ptr), ptr(ddt_ptr), int(B), int(T), int(H),
         stream_of(B_ptr))
    dA_ptr.add_(dA)


def _dtproj(dt_raw_ptr, W_ptr, bias_ptr, dt_out_ptr, B, T, H, dt_rank, stride_rb, stride_rt, stride_rr, stride_wb,
            stride_wh, stride_ob, stride_ot, stride_oh, DT_MIN=1e-3, DT_MAX=1e-1, BLOCK_H=None, BLOCK_R=None, **_):
    """dt_project_softplus_kernel (discretize_kernel.py:165-213)."""
    if (int(B), int(T), int(dt_rank)) != tuple(dt_raw_ptr.shape) or tuple(W_ptr.shape) != (int(dt_rank), int(H)):
        raise ValueError("dt_project_softplus_kernel: sizes do not match the tensors")
    ops.dt_project_softplus(dt_raw_ptr, W_ptr, bias_ptr, DT_MIN, DT_MAX, out=dt_out_ptr)


discretize_kernel = types.SimpleNamespace(
    zoh_discretize_diag_kernel=_Launchable("zoh_discretize_diag_kernel", _zoh(torch.float32)),
    zoh_discretize_diag_bf16_kernel=_Launchable("zoh_discretize_diag_bf16_kernel", _zoh(torch.bfloat16)),
    zoh_discretize_bwd_kernel=_Launchable("zoh_discretize_bwd_kernel", _zoh_bwd),
    dt_project_softplus_kernel=_Launchable("dt_project_softplus_kernel", _dtproj),
)


# ------------------------------------------------------------- ssm_scan.py
# The host functions ssm_forward / ssm_backward (ssm_scan.py:239-289) map to the
# fused one-launch operators; the individual kernels they launch map to the
# blocked multi-pass entry points (tssm_ssm_fwd_local, ...), which keep the
# reference's intermediate layouts so the launches compose as the reference's do.
def _contig_f32(*ts):
    ops._cuda(*ts)
    for t in ts:
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("the ssm_scan kernels take contiguous f32 tensors")


def _fwd_local(u_ptr, A_ptr, B_ptr, loc_a_ptr, loc_x_ptr, carry_ptr, B, L, H, BLK, NBLK, **_):
    _contig_f32(u_ptr, A_ptr, B_ptr, loc_a_ptr, loc_x_ptr, carry_ptr)
    call("tssm_ssm_fwd_local", ptr(u_ptr), ptr(A_ptr), ptr(B_ptr), ptr(loc_a_ptr), ptr(loc_x_ptr), ptr(carry_ptr),
         int(B), int(L), int(H), int(BLK), int(NBLK), stream_of(u_ptr))


def _carry_scan(reverse):
    def run(carry_ptr, nrows, NBLK, **_):
        _contig_f32(carry_ptr)
        if carry_ptr.numel() < 2 * int(nrows) * int(NBLK):
            raise ValueError("carry must hold 2 * nrows * NBLK values")
        call("tssm_blocked_carry_scan", ptr(carry_ptr), int(nrows), int(NBLK), 1 if reverse else 0,
             stream_of(carry_ptr))
    return run


def _fwd_apply(loc_a_ptr, loc_x_ptr, carry_ptr, h_out_ptr, B, L, H, BLK, NBLK, **_):
    _contig_f32(loc_a_ptr, loc_x_ptr, carry_ptr, h_out_ptr)
    call("tssm_ssm_fwd_apply", ptr(loc_a_ptr), ptr(loc_x_ptr), ptr(carry_ptr), ptr(h_out_ptr), int(B), int(L), int(H),
         int(BLK), int(NBLK), stream_of(h_out_ptr))


def _output(h_ptr, C_ptr, D_ptr, u_ptr, y_ptr, B, L, H, BLK=None, **_):
    _contig_f32(h_ptr, C_ptr, D_ptr, u_ptr, y_ptr)
    call("tssm_ssm_output", ptr(h_ptr), ptr(C_ptr), ptr(D_ptr), ptr(u_ptr), ptr(y_ptr), int(B), int(L), int(H),
         stream_of(y_ptr))


def _bwd_local(A_ptr, C_ptr, dY_ptr, loc_a_ptr, loc_dh_ptr, carry_ptr, B, L, H, BLK, NBLK, **_):
    _contig_f32(A_ptr, C_ptr, dY_ptr, loc_a_ptr, loc_dh_ptr, carry_ptr)
    call("tssm_ssm_bwd_local", ptr(A_ptr), ptr(C_ptr), ptr(dY_ptr), ptr(loc_a_ptr), ptr(loc_dh_ptr), ptr(carry_ptr),
         int(B), int(L), int(H), int(BLK), int(NBLK), stream_of(A_ptr))


def _bwd_apply(loc_a_ptr, loc_dh_ptr, carry_ptr, u_ptr, A_ptr, B_ptr, h_ptr, dY_ptr, du_ptr, dA_ptr, dB_ptr,
               dC_ptr, B, L, H, BLK, NBLK, **_):
    _contig_f32(loc_a_ptr, loc_dh_ptr, carry_ptr, u_ptr, A_ptr, B_ptr, h_ptr, dY_ptr, du_ptr, dA_ptr, dB_ptr,
                dC_ptr)
    call("tssm_ssm_bwd_apply", ptr(loc_a_ptr), ptr(loc_dh_ptr), ptr(carry_ptr), ptr(u_ptr), ptr(A_ptr), ptr(B_ptr),
         ptr(h_ptr), ptr(dY_ptr), ptr(du_ptr), ptr(dA_ptr), ptr(dB_ptr), ptr(dC_ptr), int(B), int(L), int(H),
         int(BLK), int(NBLK), stream_of(u_ptr))


ssm_scan = types.SimpleNamespace(
    ssm_forward=ops.ssm_forward, ssm_backward=ops.ssm_backward,
    ssm_fwd_local_kernel=_Launchable("ssm_fwd_local_kernel", _fwd_local),
    ssm_carry_scan_kernel=_Launchable("ssm_carry_scan_kernel", _carry_scan(False)),
    ssm_fwd_apply_kernel=_Launchable("ssm_fwd_apply_kernel", _fwd_apply),
    ssm_output_kernel=_Launchable("ssm_output_kernel", _output),
    ssm_bwd_local_kernel=_Launchable("ssm_bwd_local_kernel", _bwd_local),
    ssm_bwd_carry_scan_kernel=_Launchable("ssm_bwd_carry_scan_kernel", _carry_scan(True)),
    ssm_bwd_apply_kernel=_Launchable("ssm_bwd_apply_kernel", _bwd_apply),
)


# ------------------------------------------------------------- multihead_ssm_kernel.py
def _mh_dtype(*ts):
    d = ts[0].dtype
    if d not in (torch.float32, torch.bfloat16) or any(t.dtype != d for t in ts):
        raise ValueError("u, B and C must share a dtype, f32 or bf16")
    return F32 if d == torch.float32 else BF16


def _mh_local(u_ptr, A_log_ptr, B_ptr, C_ptr, dt_ptr, loc_a_ptr, loc_x_ptr, carry_ptr, B, L, H, n_heads, head_dim,
              stride_ub, stride_ul, stride_uh, stride_alh, stride_alp, stride_Bb, stride_Bl, stride_Bh, stride_Bp,
              stride_Cb, stride_Cl, stride_Ch, stride_Cp, stride_db, stride_dl, stride_dh, BLK_L=256, NBLK=1,
              HEAD_DIM=None, **_):
    """multihead_ssm_fwd_local_kernel (multihead_ssm_kernel.py:19-102)."""
    ops._cuda(u_ptr, A_log_ptr, B_ptr, dt_ptr, loc_a_ptr, loc_x_ptr, carry_ptr)
    if (stride_uh, stride_alp, stride_Bp) != (1, 1, 1):
        raise ValueError("the head-dim strides must be 1 (as the reference's loads assume)")
    if int(H) != int(n_heads) * int(head_dim):
        raise ValueError("H must be n_heads * head_dim")
    for t in (loc_a_ptr, loc_x_ptr, carry_ptr):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("loc_a, loc_x and carry must be contiguous f32")
    dt = _f32(dt_ptr)
    dts = (dt_ptr.stride(0), dt_ptr.stride(1), dt_ptr.stride(2)) if dt is not dt_ptr else \
        (stride_db, stride_dl, stride_dh)
    call("tssm_mh_fwd_local", ptr(u_ptr), ptr(_f32(A_log_ptr)), ptr(B_ptr), ptr(dt), ptr(loc_a_ptr), ptr(loc_x_ptr),
         ptr(carry_ptr), int(B), int(L), int(n_heads), int(head_dim), int(stride_ub), int(stride_ul),
         int(stride_alh), int(stride_Bb), int(stride_Bl), int(stride_Bh), *(int(v) for v in dts), int(BLK_L),
         int(NBLK), _mh_dtype(u_ptr, B_ptr), stream_of(u_ptr))


def _mh_output(loc_a_ptr, loc_x_ptr, carry_ptr, C_ptr, D_ptr, u_ptr, y_ptr, B, L, H, n_heads, head_dim,
               stride_ub, stride_ul, stride_uh, stride_Cb, stride_Cl, stride_Ch, stride_Cp, BLK_L=256, NBLK=1,
               HEAD_DIM=None, **_):
    """multihead_ssm_output_kernel (multihead_ssm_kernel.py:120-187); y is
    [B, L, H] contiguous with each head's readout on every position of its
    slice."""
    ops._cuda(loc_a_ptr, loc_x_ptr, carry_ptr, C_ptr, D_ptr, u_ptr, y_ptr)
    if (stride_uh, stride_Cp) != (1, 1) or int(H) != int(n_heads) * int(head_dim):
        raise ValueError("head-dim strides must be 1 and H = n_heads * head_dim")
    if y_ptr.dtype != u_ptr.dtype or not y_ptr.is_contiguous():
        raise ValueError("y must be contiguous in u's dtype")
    call("tssm_mh_output", ptr(loc_a_ptr), ptr(loc_x_ptr), ptr(carry_ptr), ptr(C_ptr), ptr(_f32(D_ptr).contiguous()),
         ptr(u_ptr), ptr(y_ptr), int(B), int(L), int(n_heads), int(head_dim), int(stride_ub), int(stride_ul),
         int(stride_Cb), int(stride_Cl), int(stride_Ch), int(BLK_L), int(NBLK), _mh_dtype(u_ptr, C_ptr),
         stream_of(y_ptr))


multihead_ssm_kernel = types.SimpleNamespace(
    multihead_ssm_fwd_local_kernel=_Launchable("multihead_ssm_fwd_local_kernel", _mh_local),
    multihead_ssm_carry_scan_kernel=_Launchable("multihead_ssm_carry_scan_kernel", _carry_scan(False)),
    multihead_ssm_output_kernel=_Launchable("multihead_ssm_output_kernel", _mh_output),
)


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


def _ring(ring_V_ptr, ring_M_ptr, ring_tau_ptr, ring_head_ptr, v_new_ptr, m_new_ptr, tau_new_ptr, h_ptr, Abar_ptr,
          Bbar_ptr, C_ptr, D_ptr, y_ptr, B, H, K, stride_rb, stride_rk, stride_rh, stride_vb, stride_vh, stride_hb,
          stride_hh, stride_cb, stride_ch, BLOCK_H=128, KRING=None, **_):
    """streaming_interp_then_ssm_kernel (streaming_inference_kernel.py:74-156),
    race-free: one CTA owns each stream's ring head.  BLOCK_H is the feature
    tile over which mask sums decide "observed", as in the reference."""
    if KRING is not None and int(KRING) != int(K) + 1:
        raise ValueError("KRING must be K + 1")
    if tuple(ring_V_ptr.shape) != (int(B), int(K) + 1, int(H)):
        raise ValueError("ring_V must be [B, K+1, H]")
    ops.streaming_interp_then_ssm(ring_V_ptr, ring_M_ptr, ring_tau_ptr, ring_head_ptr, v_new_ptr, m_new_ptr,
                                  tau_new_ptr, h_ptr, Abar_ptr, Bbar_ptr, C_ptr, D_ptr, y=y_ptr, BLOCK_H=BLOCK_H)


def _pool(h_ptr, W_ptr, bias_ptr, out_ptr, B, T, H, stride_b, stride_t, stride_h, BLOCK_H=None, BLOCK_T=None, **_):
    """mean_pool_logit_kernel (streaming_inference_kernel.py:159-194)."""
    ops._cuda(h_ptr, W_ptr, bias_ptr, out_ptr)
    if tuple(h_ptr.shape) != (int(B), int(T), int(H)) or out_ptr.dtype != torch.float32 or \
            not out_ptr.is_contiguous() or out_ptr.numel() < int(B):
        raise ValueError("mean_pool_logit_kernel: h must be [B,T,H] and out a contiguous f32 [B]")
    out_ptr[:int(B)].copy_(ops.mean_pool_logit(h_ptr, W_ptr, bias_ptr))


streaming_inference_kernel = types.SimpleNamespace(
    streaming_ssm_inplace_kernel=_Launchable("streaming_ssm_inplace_kernel", _stream(torch.float32)),
    streaming_ssm_inplace_bf16_kernel=_Launchable("streaming_ssm_inplace_bf16_kernel", _stream(torch.bfloat16)),
    streaming_interp_then_ssm_kernel=_Launchable("streaming_interp_then_ssm_kernel", _ring),
    mean_pool_logit_kernel=_Launchable("mean_pool_logit_kernel", _pool),
)

# Reference kernels deliberately not provided: residual_add_kernel and
# dropout_residual_kernel (multihead_ssm_kernel.py:190-222), layernorm_kernel,
# layernorm_bwd_kernel, swiglu_kernel, swiglu_bwd_kernel
# (fused_ssm_interp.py:104-217) and masked_fill_zero_kernel
# (streaming_inference_kernel.py:197-214) are model glue outside the SSM hot
# path; the @triton.jit combine helpers (_combine, _combine_fwd, _combine_bwd,
# _scan_combine) are device functions, not launches.
NOT_PROVIDED = ("residual_add_kernel", "dropout_residual_kernel", "layernorm_kernel", "layernorm_bwd_kernel",
                "swiglu_kernel", "swiglu_bwd_kernel", "masked_fill_zero_kernel",
                "_combine", "_combine_fwd", "_combine_bwd", "_scan_combine")

__all__ = ["discretize_kernel", "ssm_scan", "multihead_ssm_kernel", "fused_interp_kernel", "fused_ssm_interp",
           "streaming_inference_kernel", "NOT_PROVIDED"]
