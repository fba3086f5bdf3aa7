"""Benchmark of the selective-SSM hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2]

Default workload: config 2 of the reference's benchmark set (multi-head
chunked scan, B=16 H=8 P=64 N=64 L=8192, bf16 inputs, f32 state), one step =
one full pass over one batch.  Under torchrun each rank runs its own batch
(weak scaling, no collective on the data path); the time is the max over ranks.
Prints ONE JSON line on rank 0.
"""
import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "state-updates/sec (B*L*H*P*N)"
UNIT = "state-updates/s"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU through NVML every
    `period` seconds on a background thread (reading only)."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index, period=0.02):
        self.samples, self.reasons, self.ok = [], set(), False
        self.period = period
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # no NVML: report what we can
            self.err = str(e)
            self.max_mhz = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                m = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if m & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": len(self.samples)}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# --------------------------------------------------------------------------- helpers
def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def read_profile_traffic(name):
    """DRAM bytes per launch recorded from an ncu capture in profiles/<name>
    (line `dram_bytes_per_launch: <int>`), or None."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(p):
            if line.strip().startswith("dram_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def time_loop(fn, steps, stream):
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(steps):
        fn()
    ev1.record(stream)
    torch.cuda.synchronize()
    return ev0.elapsed_time(ev1) / 1e3          # seconds for all steps


# --------------------------------------------------------------------------- CPU baseline
def cpu_ssd_rate(Bt, H, P, N, L_sample, seconds, seed=0):
    """Time the CPU oracle (torch, all host threads) on [Bt, L_sample] slices of
    the config until `seconds` have passed; return (updates/s, threads, sample)."""
    import oracle
    from triton_ssm_b200 import workloads
    torch.set_num_threads(os.cpu_count() or 1)
    inp = workloads.ssd_inputs(Bt, L_sample, H, P, N, "cpu", seed)
    t0 = time.perf_counter()
    n = 0
    while True:
        oracle.ssd_scan_chunked(inp["x"], inp["dt"], inp["A_log"], inp["B"], inp["C"], inp["D"],
                                chunk=256, return_state=False)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    upd = n * workloads.ssd_updates(Bt, L_sample, H, P, N)
    return upd / el, torch.get_num_threads(), "oracle.ssd_scan_chunked on B=%d H=%d L=%d slices x%d (%.1f s)" % (
        Bt, H, L_sample, n, el)


# --------------------------------------------------------------------------- arms
def run_reference(args, rank, world):
    """The reference arm: the CPU restatement of the reference's path (the
    oracle port), all host threads, on bounded samples of the same workload."""
    if rank != 0:
        return None
    from triton_ssm_b200 import workloads
    c = workloads.C2
    # size each step so that (warmup + steps) samples take about a minute in total
    budget = float(os.environ.get("TSSM_REF_BUDGET_S", "60"))
    probe_rate, threads, _ = cpu_ssd_rate(c["Bt"], c["H"], c["P"], c["N"], 256, 0.5)
    per_step = budget / max(1, args.steps + args.warmup)
    L_s = int(max(64, min(c["L"], per_step * probe_rate / (c["Bt"] * c["H"] * c["P"] * c["N"]))))
    L_s = max(64, (L_s // 64) * 64)
    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    inp = workloads.ssd_inputs(c["Bt"], L_s, c["H"], c["P"], c["N"], "cpu", 0)
    f = lambda: oracle.ssd_scan_chunked(inp["x"], inp["dt"], inp["A_log"], inp["B"], inp["C"], inp["D"],
                                        chunk=256, return_state=False)
    for _ in range(args.warmup):
        f()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        f()
    el = time.perf_counter() - t0
    upd = workloads.ssd_updates(c["Bt"], L_s, c["H"], c["P"], c["N"]) * args.steps
    v = upd / el
    sample = "oracle.ssd_scan_chunked (torch CPU) on B=%d H=%d P=%d N=%d, L=%d of %d per step" % (
        c["Bt"], c["H"], c["P"], c["N"], L_s, c["L"])
    return {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": "config2: multi-head chunked scan B16 H8 P64 N64 L8192 (sampled on CPU)",
                   "global_batch": c["Bt"], "seq_len": c["L"], "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_ours_c2(args, rank, world, local):
    import triton_ssm_b200 as ts
    from triton_ssm_b200 import workloads
    from triton_ssm_b200.host import SSDHostPipeline
    ts.load_library()
    dev = torch.device("cuda", local)
    c = workloads.C2
    Bt, L, H, P, N = args.batch or c["Bt"], c["L"], c["H"], c["P"], c["N"]
    inp = workloads.ssd_inputs(Bt, L, H, P, N, dev, seed=1234 + rank)
    y = torch.empty_like(inp["x"])
    stream = torch.cuda.current_stream(dev)
    step = lambda: ts.multihead_ssm(inp["x"], inp["A_log"], inp["B"], inp["C"], inp["dt"], inp["D"], y=y)

    for _ in range(args.warmup):
        step()
    ts.check_device_status()
    barrier(world)
    # keep the GPU busy for >= 1 s before timing so the clock samples reflect load
    t_end = time.perf_counter() + (0.0 if args.no_soak else 1.0)
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        while time.perf_counter() < t_end:
            for _ in range(20):
                step()
            torch.cuda.synchronize()
        barrier(world)
        el = time_loop(step, args.steps, stream)
    ts.check_device_status()
    el = max_over_ranks(el, world)
    t_step = el / args.steps
    upd = workloads.ssd_updates(Bt, L, H, P, N)
    value = world * upd / t_step
    alg_bytes = workloads.ssd_bytes(Bt, L, H, P, N)
    peak, peak_kind = peaks()
    achieved = alg_bytes / t_step / 1e9

    # ---- end to end through the public host-buffer API (pinned host memory)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e_c2(inp, y, Bt, L, H, P, N, dev, args, world, upd)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        r, thr, sample = cpu_ssd_rate(Bt, H, P, N, 512, args.cpu_seconds)
        cpu = {"value": r, "unit": UNIT, "cores": thr, "kind": "port", "sample": sample}

    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config2: multi-head chunked scan (SSD state) B%d H8 P64 N64 L8192, "
                               "chunk 256 (kernel tile 64), Euler B, bf16 in / f32 state" % Bt,
                   "global_batch": Bt * world, "seq_len": L, "heads": H, "head_dim": P, "d_state": N,
                   "parallelism": "batch x head, %d independent rank(s)" % world,
                   "l2": "inputs (%d MB/step) larger than the 126 MB L2; no flush" % (alg_bytes // 2**20)},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": alg_bytes,
                     "traffic": read_profile_traffic("ssd_chunk_scan_c2.md"),
                     "kernel": "ssd_chunk_scan_kernel<64,false>"},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }


def run_e2e_c2(inp, y, Bt, L, H, P, N, dev, args, world, upd):
    from triton_ssm_b200.host import SSDHostPipeline
    e2e_steps = max(3, min(args.steps, 20))
    host = {k: v.cpu().pin_memory() for k, v in inp.items()}
    y_h = torch.empty(y.shape, dtype=y.dtype).pin_memory()
    pipe = SSDHostPipeline(Bt, L, H, P, N, dev, nslices=8)
    run = lambda: pipe(host["x"], host["dt"], host["A_log"], host["B"], host["C"], host["D"], y_h)
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    barrier(world)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(pipe.s_h2d)
    for _ in range(e2e_steps):
        run()
    pipe.s_h2d.wait_stream(pipe.s_d2h)
    ev1.record(pipe.s_h2d)
    torch.cuda.synchronize()
    e2e_t = max_over_ranks(ev0.elapsed_time(ev1) / 1e3 / e2e_steps, world)
    # spot-check the host result against the device result
    if not torch.equal(y_h.to(dev), y):
        raise RuntimeError("host-pipeline output differs from the device run")
    return {"value": world * upd / e2e_t, "unit": UNIT, "h2d_bytes_per_step": pipe.h2d_bytes(),
            "d2h_bytes_per_step": pipe.d2h_bytes(), "ms_per_step": e2e_t * 1e3, "steps": e2e_steps,
            "gpu_launches": len(pipe.slices) * e2e_steps,
            "path": "triton_ssm_b200.host.SSDHostPipeline (pinned host buffers, 8 batch slices)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-soak", action="store_true", help="skip the 1 s pre-timing load")
    ap.add_argument("--batch", type=int, default=None, help="override the batch (profiling runs)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    rank, world, local = dist_env()
    if args.impl == "reference":
        out = run_reference(args, rank, world)
        if out is not None:
            print(json.dumps(out), flush=True)
        return 0
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        out = run_ours_c2(args, rank, world, local)
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
