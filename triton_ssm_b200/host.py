"""Host-buffer entry points: run an operator on pinned host tensors, with the
host->device copies, the kernel and the device->host copy of the result
overlapped across batch slices on three CUDA streams (two copy engines and
the SMs work at once).  Device buffers are allocated once per pipeline object
and reused.
"""
import torch

from . import ops


class SSDHostPipeline:
    """``multihead_ssm`` (mode "ssd") over pinned host inputs and output.

    The batch is cut into ``nslices`` slices; slice i+1 is copied in while
    slice i is scanned and slice i-1 is copied out.  Two device buffer sets
    alternate between slices.
    """

    def __init__(self, Bt, L, H, P, N, device, nslices=4, bdisc="euler"):
        self.shape = (Bt, L, H, P, N)
        self.device = torch.device(device)
        self.bdisc = bdisc
        nslices = max(1, min(nslices, Bt))
        step = (Bt + nslices - 1) // nslices
        self.slices = [(b, min(Bt, b + step)) for b in range(0, Bt, step)]
        m = step
        dev = self.device
        bf = torch.bfloat16
        self.bufs = [dict(x=torch.empty(m, L, H * P, device=dev, dtype=bf),
                          dt=torch.empty(m, L, H, device=dev, dtype=torch.float32),
                          B=torch.empty(m, L, H, N, device=dev, dtype=bf),
                          C=torch.empty(m, L, H, N, device=dev, dtype=bf),
                          y=torch.empty(m, L, H * P, device=dev, dtype=bf)) for _ in range(2)]
        self.A_log = torch.empty(H, device=dev)
        self.D = torch.empty(H * P, device=dev)
        self.s_h2d = torch.cuda.Stream(dev)
        self.s_comp = torch.cuda.Stream(dev)
        self.s_d2h = torch.cuda.Stream(dev)
        self.ev_in = [torch.cuda.Event() for _ in range(2)]
        self.ev_comp = [torch.cuda.Event() for _ in range(2)]
        self.ev_out = [torch.cuda.Event() for _ in range(2)]
        self.launches = 0
        self._slot = 0      # slices issued so far, across calls (buffer reuse hazards span calls)

    def h2d_bytes(self):
        Bt, L, H, P, N = self.shape
        return Bt * L * H * P * 2 + 2 * Bt * L * H * N * 2 + Bt * L * H * 4 + H * 4 + H * P * 4

    def d2h_bytes(self):
        Bt, L, H, P, N = self.shape
        return Bt * L * H * P * 2

    def __call__(self, x, dt, A_log, B, C, D, y):
        """All arguments are pinned host tensors; ``y`` receives the result.
        Work is queued on the pipeline's streams; the call returns once the
        last copy is queued (synchronise on ``self.s_d2h`` to wait)."""
        with torch.cuda.stream(self.s_h2d):
            for k in range(min(2, self._slot)):
                self.s_h2d.wait_event(self.ev_comp[k])          # previous call's kernels are done
            self.A_log.copy_(A_log, non_blocking=True)
            self.D.copy_(D, non_blocking=True)
        for (b0, b1) in self.slices:
            i = self._slot
            self._slot += 1
            k = i & 1
            buf = self.bufs[k]
            n = b1 - b0
            with torch.cuda.stream(self.s_h2d):
                if i >= 2:
                    self.s_h2d.wait_event(self.ev_comp[k])      # inputs of slice i-2 consumed
                buf["x"][:n].copy_(x[b0:b1], non_blocking=True)
                buf["dt"][:n].copy_(dt[b0:b1], non_blocking=True)
                buf["B"][:n].copy_(B[b0:b1], non_blocking=True)
                buf["C"][:n].copy_(C[b0:b1], non_blocking=True)
                self.ev_in[k].record(self.s_h2d)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(self.ev_in[k])
                if i >= 2:
                    self.s_comp.wait_event(self.ev_out[k])      # y of slice i-2 copied out
                ops.multihead_ssm(buf["x"][:n], self.A_log, buf["B"][:n], buf["C"][:n], buf["dt"][:n],
                                  self.D, bdisc=self.bdisc, y=buf["y"][:n])
                self.launches += 1
                self.ev_comp[k].record(self.s_comp)
            with torch.cuda.stream(self.s_d2h):
                self.s_d2h.wait_event(self.ev_comp[k])
                y[b0:b1].copy_(buf["y"][:n], non_blocking=True)
                self.ev_out[k].record(self.s_d2h)
        return y
