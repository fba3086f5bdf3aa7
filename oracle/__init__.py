"""CPU oracle for the selective-SSM hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU (fp32 by default, fp64 on
request), the arithmetic of the reference's Triton kernels (Triton-SSM), one
function per kernel, each citing the reference ``file:line`` it follows.  It is
pinned against golden fixtures in ``tests/golden/`` that were produced by the
reference's own kernels (see ``tests/golden/make_golden.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline.  The product path
(``triton_ssm_b200``) never calls into it: it has no CPU fallback.
"""
from .discretize import zoh_discretize, zoh_discretize_bwd, expm1_ref, dt_project_softplus, zoh_discretize_dt
from .scan import ssm_forward, ssm_backward, selective_scan
from .multihead import (ssd_scan, ssd_scan_chunked, multihead_diag, ssd_sharded_compose,
                        ssd_slice_scan, ssd_carry_fixup)
from .interp import (time_aware_interp, interp_neighbors_index, interp_neighbors_time,
                     interp_gather, interp_ssm_step, interp_ssm, linspace_queries)
from .streaming import (streaming_ssm_inplace, streaming_step, ring_interp_then_ssm, mean_pool_logit)

__all__ = [
    "zoh_discretize", "zoh_discretize_bwd", "expm1_ref", "dt_project_softplus", "zoh_discretize_dt",
    "ssm_forward", "ssm_backward", "selective_scan",
    "ssd_scan", "ssd_scan_chunked", "multihead_diag", "ssd_sharded_compose", "ssd_slice_scan",
    "ssd_carry_fixup",
    "time_aware_interp", "interp_neighbors_index", "interp_neighbors_time",
    "interp_gather", "interp_ssm_step", "interp_ssm", "linspace_queries",
    "streaming_ssm_inplace", "streaming_step", "ring_interp_then_ssm", "mean_pool_logit",
]
