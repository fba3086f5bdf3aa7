"""The C ABI: the library builds, loads without a GPU, and exports every entry
point declared in include/*.h with the argument list the binding uses."""
import glob
import os
import re

import pytest

from conftest import ROOT


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(tssm_\w+)\s*\(", src))
    return names


def _arg_count(name):
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        m = re.search(r"\b%s\s*\(([^)]*)\)" % name, src)
        if m:
            body = m.group(1).strip()
            return 0 if body in ("", "void") else body.count(",") + 1
    raise KeyError(name)


def test_library_exports_every_declared_symbol():
    from triton_ssm_b200 import _lib
    lib = _lib.load_library()
    declared = _declared()
    assert declared, "no declarations found"
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_signatures_match_header():
    from triton_ssm_b200 import _lib
    for name in _declared():
        assert name in _lib.SIGNATURES, name
        assert len(_lib.SIGNATURES[name][0]) == _arg_count(name), name


def test_status_strings_and_errors_without_gpu():
    from triton_ssm_b200 import _lib
    lib = _lib.load_library()
    assert lib.tssm_version() >= 100
    assert lib.tssm_status_string(0) == b"ok"
    assert lib.tssm_status_string(1) == b"invalid argument"


def test_ops_refuse_cpu_tensors():
    import torch
    import triton_ssm_b200 as ts
    x = torch.zeros(2, 3, 4)
    with pytest.raises(ValueError):
        ts.ssm_forward(x, x, x, x, torch.zeros(4))


def test_compat_namespaces_mirror_reference_names():
    from triton_ssm_b200 import compat
    assert hasattr(compat.discretize_kernel, "zoh_discretize_diag_kernel")
    assert hasattr(compat.discretize_kernel, "zoh_discretize_diag_bf16_kernel")
    assert hasattr(compat.fused_interp_kernel, "fused_interp_fp16_kernel")
    assert hasattr(compat.fused_ssm_interp, "fused_interp_ssm_step_kernel")
    assert hasattr(compat.streaming_inference_kernel, "streaming_ssm_inplace_bf16_kernel")
    assert callable(compat.ssm_scan.ssm_forward)
    # kernel objects are launched with [grid]
    fn = compat.discretize_kernel.zoh_discretize_diag_kernel[(1, 1, 1)]
    assert callable(fn)


def test_streaming_ring_refuses_cpu():
    import torch
    import triton_ssm_b200 as ts
    with pytest.raises(ValueError):
        ts.StreamingRing(2, 8, 3, torch.ones(8), torch.ones(8), torch.ones(8), device="cpu")
