"""Host-buffer entry points: run an operator on pinned host tensors, with the
host->device copies, the kernel and the device->host copy of the result
overlapped across batch slices on three CUDA streams (two copy engines and
the SMs work at once).  Device buffers are allocated once per pipeline object
and reused.
"""
import os

import torch

from . import ops


def gpu_numa_node(device):
    """NUMA node of the GPU's PCI device (sysfs), or None where the platform
    does not say (single-node hosts report -1)."""
    props = torch.cuda.get_device_properties(torch.device(device))
    bus = "%04x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
    try:
        with open("/sys/bus/pci/devices/%s/numa_node" % bus) as f:
            node = int(f.read().strip())
    except (OSError, ValueError):
        return None
    return node if node >= 0 else None


def parse_cpulist(text):
    """CPU ids of a kernel cpulist string ("0-7,16-23")."""
    cpus = set()
    for part in filter(None, text.strip().split(",")):
        lo, _, hi = part.partition("-")
        cpus.update(range(int(lo), int(hi or lo) + 1))
    return cpus


def node_cpus(node):
    """CPU ids of a NUMA node (empty when sysfs does not list it)."""
    try:
        with open("/sys/devices/system/node/node%d/cpulist" % node) as f:
            return parse_cpulist(f.read())
    except OSError:
        return set()


def gpu_ideal_cpus(device):
    """The CPUs NVML reports as nearest the GPU (a read-only query), or an
    empty set when NVML is unavailable."""
    try:
        import pynvml
    except ImportError:
        return set()
    props = torch.cuda.get_device_properties(torch.device(device))
    bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
    cpus = set()
    try:
        pynvml.nvmlInit()
        try:
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
            for w, mask in enumerate(words):
                cpus.update(64 * w + i for i in range(64) if (int(mask) >> i) & 1)
        finally:
            pynvml.nvmlShutdown()
    except pynvml.NVMLError:
        return set()
    return cpus


def bind_host_to_gpu(device):
    """Restrict this process's CPUs to those nearest the GPU -- its NUMA node's
    (sysfs), else the set NVML reports -- so pinned buffers allocated (first
    touched) afterwards sit in the memory nearest the GPU's PCIe root and host
    copies do not cross the inter-socket link.  Returns {"numa_node", "cpus",
    "source"} or None when neither source narrows the allowed CPUs (the
    affinity is then left as it was)."""
    allowed = set(os.sched_getaffinity(0))
    node = gpu_numa_node(device)
    cpus, source = (node_cpus(node) & allowed, "sysfs") if node is not None else (set(), None)
    if not cpus:
        cpus, source = gpu_ideal_cpus(device) & allowed, "nvml"
    if not cpus or cpus == allowed:
        return None
    os.sched_setaffinity(0, cpus)
    return {"numa_node": node, "cpus": len(cpus), "source": source}


def pinned_copy_gbs(device, nbytes=256 << 20, reps=4):
    """(host->device, device->host) GB/s of one pinned buffer of `nbytes`,
    timed with CUDA events on a side stream (the best of `reps` copies each)."""
    dev = torch.device(device)
    h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    s = torch.cuda.Stream(dev)
    best = []
    for direction in ("h2d", "d2h"):
        times = []
        with torch.cuda.stream(s):
            for _ in range(reps + 1):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(s)
                if direction == "h2d":
                    d.copy_(h, non_blocking=True)
                else:
                    h.copy_(d, non_blocking=True)
                e1.record(s)
                e1.synchronize()
                times.append(e0.elapsed_time(e1) / 1e3)
        best.append(nbytes / min(times[1:]) / 1e9)
    return best[0], best[1]


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
