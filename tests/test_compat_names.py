"""The kernel-level drop-in is complete: every @triton.jit kernel that the
reference's six files launch resolves in triton_ssm_b200.compat to a
launchable shim, except the model glue the compat module lists as not
provided.  (CPU: nothing is launched.)"""
import pytest

# (reference module, @triton.jit name, file:line of its definition)
REFERENCE_JIT = [
    ("discretize_kernel", "zoh_discretize_diag_kernel", "discretize_kernel.py:16"),
    ("discretize_kernel", "zoh_discretize_diag_bf16_kernel", "discretize_kernel.py:61"),
    ("discretize_kernel", "zoh_discretize_bwd_kernel", "discretize_kernel.py:98"),
    ("discretize_kernel", "dt_project_softplus_kernel", "discretize_kernel.py:166"),
    ("fused_interp_kernel", "fused_time_aware_interp_kernel", "fused_interp_kernel.py:10"),
    ("fused_interp_kernel", "fused_interp_bf16_kernel", "fused_interp_kernel.py:104"),
    ("fused_interp_kernel", "fused_interp_fp16_kernel", "fused_interp_kernel.py:187"),
    ("fused_ssm_interp", "_combine_fwd", "fused_ssm_interp.py:7"),
    ("fused_ssm_interp", "fused_interp_ssm_step_kernel", "fused_ssm_interp.py:12"),
    ("fused_ssm_interp", "layernorm_kernel", "fused_ssm_interp.py:105"),
    ("fused_ssm_interp", "layernorm_bwd_kernel", "fused_ssm_interp.py:134"),
    ("fused_ssm_interp", "swiglu_kernel", "fused_ssm_interp.py:174"),
    ("fused_ssm_interp", "swiglu_bwd_kernel", "fused_ssm_interp.py:194"),
    ("multihead_ssm_kernel", "_scan_combine", "multihead_ssm_kernel.py:15"),
    ("multihead_ssm_kernel", "multihead_ssm_fwd_local_kernel", "multihead_ssm_kernel.py:20"),
    ("multihead_ssm_kernel", "multihead_ssm_carry_scan_kernel", "multihead_ssm_kernel.py:106"),
    ("multihead_ssm_kernel", "multihead_ssm_output_kernel", "multihead_ssm_kernel.py:121"),
    ("multihead_ssm_kernel", "residual_add_kernel", "multihead_ssm_kernel.py:191"),
    ("multihead_ssm_kernel", "dropout_residual_kernel", "multihead_ssm_kernel.py:205"),
    ("ssm_scan", "_combine", "ssm_scan.py:13"),
    ("ssm_scan", "ssm_fwd_local_kernel", "ssm_scan.py:18"),
    ("ssm_scan", "ssm_carry_scan_kernel", "ssm_scan.py:54"),
    ("ssm_scan", "ssm_fwd_apply_kernel", "ssm_scan.py:69"),
    ("ssm_scan", "ssm_output_kernel", "ssm_scan.py:102"),
    ("ssm_scan", "_combine_bwd", "ssm_scan.py:130"),
    ("ssm_scan", "ssm_bwd_local_kernel", "ssm_scan.py:136"),
    ("ssm_scan", "ssm_bwd_carry_scan_kernel", "ssm_scan.py:174"),
    ("ssm_scan", "ssm_bwd_apply_kernel", "ssm_scan.py:189"),
    ("streaming_inference_kernel", "streaming_ssm_inplace_kernel", "streaming_inference_kernel.py:7"),
    ("streaming_inference_kernel", "streaming_ssm_inplace_bf16_kernel", "streaming_inference_kernel.py:41"),
    ("streaming_inference_kernel", "streaming_interp_then_ssm_kernel", "streaming_inference_kernel.py:75"),
    ("streaming_inference_kernel", "mean_pool_logit_kernel", "streaming_inference_kernel.py:160"),
    ("streaming_inference_kernel", "masked_fill_zero_kernel", "streaming_inference_kernel.py:198"),
]

# The two Python host functions (ssm_scan.py:239, :267).
REFERENCE_HOST = [("ssm_scan", "ssm_forward"), ("ssm_scan", "ssm_backward")]


@pytest.mark.parametrize("module,name,where", REFERENCE_JIT, ids=[n for _, n, _ in REFERENCE_JIT])
def test_every_reference_kernel_resolves(module, name, where):
    from triton_ssm_b200 import compat
    if name in compat.NOT_PROVIDED:
        assert not hasattr(getattr(compat, module), name)
        return
    ns = getattr(compat, module)
    obj = getattr(ns, name, None)
    assert obj is not None, "%s (%s) has no shim" % (name, where)
    assert isinstance(obj, compat._Launchable), name
    fn = obj[(1,)]
    assert callable(fn) and "not part of this build" not in (fn.__doc__ or "")


@pytest.mark.parametrize("module,name", REFERENCE_HOST)
def test_reference_host_functions(module, name):
    from triton_ssm_b200 import compat, ops
    assert getattr(getattr(compat, module), name) is getattr(ops, name)


def test_not_provided_is_only_glue():
    from triton_ssm_b200 import compat
    in_scope = {n for _, n, _ in REFERENCE_JIT} - set(compat.NOT_PROVIDED)
    assert len(in_scope) == 22
    import inspect
    src = inspect.getsource(compat)
    assert "NotImplementedError" not in src
