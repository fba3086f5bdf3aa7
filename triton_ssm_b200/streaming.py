"""Long-running streams on the ring-buffer step, with checkpoint / restore.

``StreamingRing`` keeps everything a stream needs on the device -- the last
K+1 observations (values, masks, times), the ring head and the SSM state --
and advances all streams by one event per ``step`` through
``streaming_interp_then_ssm`` (``streaming_inference_kernel.py:74-156``).
``checkpoint`` copies that state to host memory, ``restore`` puts it back, so
a service can persist its streams and resume them bit for bit.
"""
import torch

from .ops import streaming_interp_then_ssm

__all__ = ["StreamingRing"]

_STATE = ("ring_V", "ring_M", "ring_tau", "ring_head", "h")
_PARAMS = ("Abar", "Bbar", "D")


class StreamingRing:
    """Bt independent streams of H features with a (K+1)-slot observation ring.

    Abar, Bbar, D [H] f32 are the (shared) step parameters.  ``block_h`` is the
    feature-tile width over which mask sums decide "observed"; it is part of
    the stream's definition and is kept in checkpoints.
    """

    def __init__(self, Bt, H, K, Abar, Bbar, D, device=None, block_h=128, h0=None):
        device = torch.device(device) if device is not None else Abar.device
        if device.type != "cuda":
            raise ValueError("StreamingRing lives on a CUDA device (no CPU fallback)")
        if K < 0 or K + 1 > 64:
            raise ValueError("StreamingRing: K must be in [0, 63]")
        f32 = dict(device=device, dtype=torch.float32)
        self.K, self.block_h = int(K), int(block_h)
        self.Abar, self.Bbar, self.D = (t.to(**f32).contiguous() for t in (Abar, Bbar, D))
        self.ring_V = torch.zeros(Bt, K + 1, H, **f32)
        self.ring_M = torch.zeros(Bt, K + 1, H, **f32)
        self.ring_tau = torch.zeros(Bt, K + 1, **f32)
        self.ring_head = torch.zeros(Bt, device=device, dtype=torch.int32)
        self.h = torch.zeros(Bt, H, **f32) if h0 is None else h0.to(**f32).clone().contiguous()
        self.steps = 0

    @property
    def shape(self):
        return tuple(self.h.shape)

    def step(self, v_new, m_new, tau_new, C, y=None):
        """Ingest one event per stream (v_new, m_new, C [Bt,H]; tau_new [Bt]) and
        return y [Bt,H]; the ring, head and state advance in place."""
        y = streaming_interp_then_ssm(self.ring_V, self.ring_M, self.ring_tau, self.ring_head, v_new, m_new,
                                      tau_new, self.h, self.Abar, self.Bbar, C, self.D, y=y, BLOCK_H=self.block_h)
        self.steps += 1
        return y

    def checkpoint(self, pin_memory=False):
        """A host copy of the streams' state and parameters (a dict of CPU tensors
        and ints); the copy is complete when this returns."""
        ck = {"K": self.K, "block_h": self.block_h, "steps": self.steps}
        for name in _STATE + _PARAMS:
            t = getattr(self, name)
            host = torch.empty(t.shape, dtype=t.dtype, pin_memory=pin_memory)
            host.copy_(t, non_blocking=pin_memory)
            ck[name] = host
        torch.cuda.current_stream(self.h.device).synchronize()
        return ck

    def restore(self, ck):
        """Put a checkpoint taken from a ring of the same shape back in place."""
        if int(ck["K"]) != self.K or int(ck["block_h"]) != self.block_h:
            raise ValueError("StreamingRing.restore: checkpoint has K=%s block_h=%s, ring has K=%d block_h=%d"
                             % (ck["K"], ck["block_h"], self.K, self.block_h))
        for name in _STATE + _PARAMS:
            dst = getattr(self, name)
            src = ck[name]
            if tuple(src.shape) != tuple(dst.shape) or src.dtype != dst.dtype:
                raise ValueError("StreamingRing.restore: %s has shape %s/%s, expected %s/%s"
                                 % (name, tuple(src.shape), src.dtype, tuple(dst.shape), dst.dtype))
            dst.copy_(src)
        self.steps = int(ck["steps"])

    def save(self, path):
        torch.save(self.checkpoint(), path)

    @classmethod
    def load(cls, path, device="cuda"):
        ck = torch.load(path, map_location="cpu", weights_only=True)
        Bt, KR, H = ck["ring_V"].shape
        ring = cls(Bt, H, KR - 1, ck["Abar"], ck["Bbar"], ck["D"], device=device, block_h=ck["block_h"])
        ring.restore(ck)
        return ring
