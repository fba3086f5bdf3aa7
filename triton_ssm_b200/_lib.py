"""ctypes binding of ``libtssm_b200.so`` (the C ABI declared in include/tssm.h).

There is no CPU fallback: every operator in this package needs this library
and a CUDA device, and raises when either is missing.
"""
import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtssm_b200.so")

F32, BF16, F16, U8 = 0, 1, 2, 3
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT = 0, 1, 2, 3, 4

_DTYPE_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16, torch.uint8: U8,
               torch.bool: U8}

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F64 = ctypes.c_double

# name -> argument types (the trailing stream is a c_void_p).  Must match include/tssm.h.
SIGNATURES = {
    "tssm_version": ([], I32),
    "tssm_status_string": ([I32], ctypes.c_char_p),
    "tssm_last_error": ([], ctypes.c_char_p),
    "tssm_zoh_discretize": ([P] * 5 + [I64] * 3 + [I64] * 8 + [I32, P], I32),
    "tssm_ssm_forward": ([P] * 7 + [I64] * 3 + [I32, P], I32),
    "tssm_selective_scan": ([P] * 8 + [I64] * 4 + [P], I32),
    "tssm_ssm_backward": ([P] * 10 + [I64] * 3 + [I32, P], I32),
    "tssm_ssm_forward_pool": ([P] * 10 + [I64] * 3 + [I32, P], I32),
    "tssm_mean_pool_logit": ([P] * 4 + [I64] * 3 + [I32, P], I32),
    "tssm_zoh_discretize_bwd": ([P] * 9 + [I64] * 3 + [P], I32),
    "tssm_dt_project_softplus": ([P] * 4 + [I64] * 4 + [F64, F64, P], I32),
    "tssm_zoh_discretize_dtproj": ([P] * 8 + [I64] * 4 + [F64, F64, P], I32),
    "tssm_streaming_inplace": ([P] * 7 + [I64] * 2 + [I64] * 3 + [I32, P], I32),
    "tssm_streaming_step": ([P] * 8 + [I64] * 4 + [I32, P], I32),
    "tssm_ring_ingest_step": ([P] * 13 + [I64] * 4 + [P], I32),
    "tssm_multihead_ssd": ([P] * 10 + [I64] * 5 + [I32, P], I32),
    "tssm_multihead_diag": ([P] * 7 + [I64] * 4 + [I32, I32, P], I32),
    "tssm_ssd_carry_fixup": ([P, P, I64, I64, P, P, P, P] + [I64] * 5 + [P], I32),
    "tssm_ssd_carry_fixup_pieces": ([P, P, I64, P, P, P, P] + [I64] * 5 + [P], I32),
    "tssm_ssd_carry_fixup_packed": ([P, I64, I64, P, P, P, P] + [I64] * 5 + [P], I32),
    "tssm_ssd_pieces_final_state": ([P, P, I64, P, P] + [I64] * 4 + [P], I32),
    "tssm_ssm_fwd_local": ([P] * 6 + [I64] * 5 + [P], I32),
    "tssm_ssm_bwd_local": ([P] * 6 + [I64] * 5 + [P], I32),
    "tssm_blocked_carry_scan": ([P, I64, I64, I32, P], I32),
    "tssm_ssm_fwd_apply": ([P] * 4 + [I64] * 5 + [P], I32),
    "tssm_ssm_output": ([P] * 5 + [I64] * 3 + [P], I32),
    "tssm_ssm_bwd_apply": ([P] * 12 + [I64] * 5 + [P], I32),
    "tssm_mh_fwd_local": ([P] * 7 + [I64] * 4 + [I64] * 9 + [I64] * 2 + [I32, P], I32),
    "tssm_mh_output": ([P] * 7 + [I64] * 4 + [I64] * 5 + [I64] * 2 + [I32, P], I32),
    "tssm_check_device_status": ([P], I32),
    "tssm_selftest_wait_timeout": ([I64, P], I32),
    "tssm_time_aware_interp": ([P] * 4 + [I64] * 3 + [I64] * 7 + [I64] * 2 + [I32, I32, P], I32),
    "tssm_interp_ssm_step": ([P] * 8 + [I64] * 3 + [I64] * 9 + [I64] * 3 + [I32, P], I32),
    "tssm_interp_ssm_workspace_size": ([I64] * 5, I64),
    "tssm_interp_ssm": ([P] * 13 + [I64] + [I64] * 7 + [I32, P], I32),
    "tssm_interp_ssm_static_scratch": ([P] * 12 + [I64] * 7 + [I32, P], I32),
}

_lib = None
_lock = threading.Lock()


class TSSMError(RuntimeError):
    pass


def load_library(path=None):
    """Load (once) and return the CUDA library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError("%s is not built: run `python -m triton_ssm_b200.build` "
                              "(or __graft_entry__.build())" % p)
        lib = ctypes.CDLL(p)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


def dtype_code(t):
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise ValueError("unsupported dtype %s" % t.dtype)


def stream_of(t):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def call(name, *args):
    """Invoke an entry point and turn a bad status into the matching exception."""
    lib = load_library()
    st = getattr(lib, name)(*args)
    if st == OK:
        return
    msg = (lib.tssm_last_error() or b"").decode(errors="replace")
    text = "%s: %s (%s)" % (name, lib.tssm_status_string(st).decode(), msg)
    if st in (ERR_INVALID, ERR_UNSUPPORTED):
        raise ValueError(text)
    if st == ERR_TIMEOUT:
        raise TimeoutError(text)
    raise TSSMError(text)
