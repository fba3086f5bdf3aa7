"""tssm_b200 — B200-native (sm_100a) selective-SSM hot path of Triton-SSM.

Operators keep the reference's names and argument order; each launches a
hand-written CUDA kernel through the C ABI in ``include/tssm.h``.
"""
from ._lib import load_library, LIB_PATH, TSSMError  # noqa: F401
from .ops import *  # noqa: F401,F403
from .ops import __all__ as _ops_all
from .streaming import StreamingRing  # noqa: F401

__all__ = ["load_library", "LIB_PATH", "TSSMError", "StreamingRing"] + list(_ops_all)
__version__ = "0.1.0"
