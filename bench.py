"""Benchmark of the selective-SSM hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2]

Default workload: config 2 of the reference's benchmark set (multi-head
chunked scan, B=16 H=8 P=64 N=64 L=8192, bf16 inputs, f32 state), one step =
one full pass over one batch.  Under torchrun each rank runs its own batch
(weak scaling, no collective on the data path); the time is the max over ranks.
Prints ONE JSON line on rank 0.

The same line carries the other configs under "configs" (--configs): config 4,
the sequence-parallel scan of L = 1,048,576 tokens sharded over all N ranks
with one NCCL all-gather of slice carries (strong scaling; its scan and its
exchange + fix-up times are also reported apart), and, on one GPU, configs 1,
3 and 5 (config 5 with steps/s and per-step latency percentiles).
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


def min_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
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


def _timed(args, world, dev, step):
    """Warm-up, >= 1 s of untimed load (so the clock samples see the GPU busy),
    then exactly args.steps timed steps; returns (seconds per step, clocks).
    With --graph the step is captured once in a CUDA graph and the timed loop
    replays it, so host-side Python overhead is not what gets measured."""
    import triton_ssm_b200 as ts
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    ts.check_device_status()
    if args.graph:
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        step = graph.replay
        step()
        torch.cuda.synchronize()
    barrier(world)
    t_end = time.perf_counter() + (0.0 if args.no_soak else 1.0)
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        while time.perf_counter() < t_end:
            for _ in range(5):
                step()
            torch.cuda.synchronize()
        barrier(world)
        el = time_loop(step, args.steps, stream)
    ts.check_device_status()
    return max_over_ranks(el, world) / args.steps, clk.summary()


def _line(args, world, metric, value, t_step, dtype, cfg, alg_bytes, kernel, profile, clocks, cpu=None,
          e2e=None, launches=None, extra=None):
    peak, peak_kind = peaks()
    achieved = alg_bytes / t_step / 1e9
    out = {
        "metric": metric, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic", "config": cfg,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": alg_bytes,
                     "traffic": read_profile_traffic(profile) if profile else None, "kernel": kernel},
        "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": launches if launches is not None else args.steps, "clocks": clocks,
    }
    if extra:
        out.update(extra)
    return out


def run_ours_c3(args, rank, world, local):
    """Config 3: fused interpolation + SSM, B32 L_obs 2048 -> L_q 4096, D256 N16, f32."""
    import triton_ssm_b200 as ts
    from triton_ssm_b200 import workloads
    dev = torch.device("cuda", local)
    c = workloads.C3
    Bt, T, Lq, Dm, N = args.batch or c["Bt"], c["T"], c["Lq"], c["D"], c["N"]
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    V = torch.randn(Bt, T, Dm, device=dev, generator=g)
    M = (torch.rand(Bt, T, Dm, device=dev, generator=g) < 0.7).to(torch.uint8)
    tau = torch.cumsum(torch.empty(Bt, T, device=dev).exponential_(1.0, generator=g), 1)
    A_log = torch.log(torch.arange(1, N + 1, device=dev, dtype=torch.float32)).repeat(Dm, 1)
    B = torch.randn(Dm, N, device=dev, generator=g) / math.sqrt(N)
    C = torch.randn(Dm, N, device=dev, generator=g) / math.sqrt(N)
    q = ts.linspace_queries(tau, Lq)
    dt = ((tau[:, -1] - tau[:, 0]) / (Lq - 1)).contiguous()
    ws = torch.empty(ts.interp_ssm_workspace_bytes(Bt, T, Dm, Lq), dtype=torch.uint8, device=dev)
    step = lambda: ts.fused_interp_ssm(V, M, tau, A_log, B, C, q=q, dt=dt, workspace=ws, return_state=True)
    t_step, clocks = _timed(args, world, dev, step)
    upd = Bt * Lq * Dm * N
    alg = Bt * T * Dm * 4 + Bt * T * Dm + Bt * T * 4 + Bt * Lq * Dm * 4 + Bt * Dm * N * 4 + 3 * Dm * N * 4
    cfg = {"workload": "config3: interpolation of irregular obs onto a regular query grid fused with an "
                       "N-state ZOH scan, B%d L_obs %d -> L_q %d, D %d, N %d, f32, mask Bernoulli(0.7) u8" %
                       (Bt, T, Lq, Dm, N),
           "global_batch": Bt * world, "seq_len": Lq, "parallelism": "batch, %d rank(s)" % world}
    return _line(args, world, METRIC, world * upd / t_step, t_step, "f32", cfg, alg,
                 "interp_table + interp_ssm_scan_chunk", "interp_ssm_c3.md", clocks,
                 launches=2 * args.steps)


def run_ours_c5(args, rank, world, local):
    """Config 5: streaming single-step update, 4096 streams, H16 P64 N64, f32 state."""
    import triton_ssm_b200 as ts
    from triton_ssm_b200 import workloads
    dev = torch.device("cuda", local)
    c = workloads.C5
    S = args.batch or c["S"]
    H, P, N = c["H"], c["P"], c["N"]
    w = workloads.stream_inputs(S, H, P, N, dev, seed=5 + rank)
    ev = w["events"]
    y = torch.empty(S, H, P, device=dev, dtype=torch.bfloat16)
    k = [0]

    def step():
        e = ev[k[0] % len(ev)]
        k[0] += 1
        ts.streaming_step(e["x"], e["dt"], w["h"], w["A_log"], e["B"], e["C"], w["D"], y=y)
    t_step, clocks = _timed(args, world, dev, step)
    # per-step latency distribution (event pairs around single steps)
    lat = []
    for _ in range(min(200, max(20, args.steps))):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        e1.synchronize()
        lat.append(e0.elapsed_time(e1))
    lat.sort()
    upd = S * H * P * N
    cfg = {"workload": "config5: streaming ZOH step, %d streams x H%d P%d N%d, f32 state in HBM, "
                       "bf16 events cycled from 16 sets" % (S, H, P, N),
           "global_batch": S * world, "seq_len": 1, "parallelism": "streams, %d rank(s)" % world,
           "l2": "state (%d MB) larger than the 126 MB L2" % (S * H * P * N * 4 // 2**20)}
    return _line(args, world, METRIC, world * upd / t_step, t_step, "f32", cfg,
                 workloads.stream_bytes(S, H, P, N), "streaming_step_kernel<bf16,16,4,true>", "streaming_step_c5.md",
                 clocks, extra={"steps_per_sec": 1.0 / t_step, "p50_step_ms": lat[len(lat) // 2],
                                "p99_step_ms": lat[int(len(lat) * 0.99) - 1]})


def run_ours_c1(args, rank, world, local):
    """Config 1: ZOH discretize + diagonal scan, B4 L1024 D64 N16 f32: the drop-in
    pair (zoh_discretize -> ssm_forward over H' = D*N) and the fused kernel."""
    import triton_ssm_b200 as ts
    dev = torch.device("cuda", local)
    Bt, L, Dm, N = 4, 1024, 64, 16
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)
    x = torch.randn(Bt, L, Dm, device=dev, generator=g)
    dt = torch.empty(Bt, L, device=dev).exponential_(1.0, generator=g).clamp_(1e-3, 10.0)
    A_log = torch.log(torch.arange(1, N + 1, device=dev, dtype=torch.float32)).repeat(Dm, 1)
    Bs = torch.randn(Bt, L, N, device=dev, generator=g) / math.sqrt(N)
    Cs = torch.randn(Bt, L, N, device=dev, generator=g) / math.sqrt(N)
    D = torch.randn(Dm, device=dev, generator=g)
    Hp = Dm * N
    B_exp = Bs[:, :, None, :].expand(Bt, L, Dm, N).reshape(Bt, L, Hp).contiguous()
    C_exp = Cs[:, :, None, :].expand(Bt, L, Dm, N).reshape(Bt, L, Hp).contiguous()
    u_exp = x[:, :, :, None].expand(Bt, L, Dm, N).reshape(Bt, L, Hp).contiguous()
    Al = A_log.reshape(-1).contiguous()
    Dz = torch.zeros(Hp, device=dev)
    if args.c1_mode == "pair":
        def step():
            Ab, Bb = ts.zoh_discretize(Al, B_exp, dt)
            ts.ssm_forward(u_exp, Ab, Bb, C_exp, Dz)
        alg = 151019520
        kern = "zoh_discretize_kernel + ssm_forward_tma_kernel"
        launches = 2 * args.steps
    elif args.c1_mode == "pool":
        # the pair with the mean-pooled logit head fused into the scan's epilogue
        Wp = torch.randn(Hp, device=dev, generator=g) / math.sqrt(Hp)
        bp = torch.zeros(1, device=dev)

        def step():
            Ab, Bb = ts.zoh_discretize(Al, B_exp, dt)
            ts.ssm_forward(u_exp, Ab, Bb, C_exp, Dz, pool=(Wp, bp))
        alg = 151019520 + Hp * 4 + 4 + Bt * 4
        kern = "zoh_discretize_kernel + ssm_forward_kernel (fused mean-pool head)"
        launches = 2 * args.steps
    else:
        step = lambda: ts.selective_scan(x, dt, A_log, Bs, Cs, D)
        alg = 2642176
        kern = "selective_scan_kernel"
        launches = args.steps
    t_step, clocks = _timed(args, world, dev, step)
    upd = Bt * L * Dm * N
    cfg = {"workload": "config1 (%s): ZOH discretize + selective scan B4 L1024 D64 N16 f32" % args.c1_mode,
           "global_batch": Bt * world, "seq_len": L, "parallelism": "batch, %d rank(s)" % world,
           "timing": "CUDA-graph replays of the step" if args.graph else "eager launches",
           "l2": ("151 MB of inputs and outputs per step (> the 126 MB L2); no flush" if args.c1_mode != "fused"
                  else "2.6 MB working set (stays in L2; latency bound)")}
    return _line(args, world, METRIC, world * upd / t_step, t_step, "f32", cfg, alg, kern, None, clocks,
                 launches=launches)


def run_ours_c1bwd(args, rank, world, local):
    """Config 1 backward: the drop-in backward pair at the config-1 forward's
    shapes (B4 L1024, H' = D*N = 1024, f32): ssm_backward (dY -> du, dA, dB, dC)
    then zoh_discretize_bwd (dAbar = dA, dBbar = dB -> dA_log, dB, ddt)."""
    import triton_ssm_b200 as ts
    dev = torch.device("cuda", local)
    Bt, L, Hp = 4, 1024, 1024
    g = torch.Generator(device=dev)
    g.manual_seed(13 + rank)
    A_log = torch.log(torch.arange(1, 17, device=dev, dtype=torch.float32)).repeat(64)
    Bc = torch.randn(Bt, L, Hp, device=dev, generator=g) / 4.0
    dt = torch.empty(Bt, L, device=dev).exponential_(1.0, generator=g).clamp_(1e-3, 10.0)
    u = torch.randn(Bt, L, Hp, device=dev, generator=g)
    C = torch.randn(Bt, L, Hp, device=dev, generator=g) / 4.0
    Ab, Bb = ts.zoh_discretize(A_log, Bc, dt)
    _, h = ts.ssm_forward(u, Ab, Bb, C, torch.zeros(Hp, device=dev))
    dY = torch.randn(Bt, L, Hp, device=dev, generator=g)

    def step():
        du, dA, dB, dC = ts.ssm_backward(u, Ab, Bb, C, h, dY)
        ts.zoh_discretize_bwd(A_log, Bc, dt, Ab, dA, dB)
    t_step, clocks = _timed(args, world, dev, step)
    n = Bt * L * Hp
    alg = n * 4 * 10 + n * 4 * 5 + Bt * L * 4 * 2 + Hp * 4 * 2   # ssm_backward 6R+4W, discretize_bwd 4R+1W
    upd = Bt * L * Hp
    cfg = {"workload": "config1 backward: ssm_backward + zoh_discretize_bwd, B4 L1024 H'=D*N=1024 f32",
           "global_batch": Bt * world, "seq_len": L, "parallelism": "batch, %d rank(s)" % world,
           "timing": "CUDA-graph replays of the step" if args.graph else "eager launches"}
    return _line(args, world, METRIC, world * upd / t_step, t_step, "f32", cfg, alg,
                 "ssm_backward_kernel + zoh_discretize_bwd_kernel", "ssm_backward_c1.md", clocks,
                 launches=2 * args.steps)


def run_ours_disc(args, rank, world, local):
    """The standalone ZOH discretisation streams at config 1's H' = D*N = 1024
    (B4 T1024, f32): zoh_discretize (read B, write Abar and Bbar: 12 B per
    element) and zoh_discretize_bwd (read B, Abar, dAbar, dBbar, write dB: 20 B
    per element, plus ddt and dA_log), each timed alone as CUDA-graph replays."""
    import copy
    import triton_ssm_b200 as ts
    dev = torch.device("cuda", local)
    Bt, T, H = args.batch or 4, 1024, 1024
    g = torch.Generator(device=dev)
    g.manual_seed(41 + rank)
    A_log = torch.log(torch.arange(1, 17, device=dev, dtype=torch.float32)).repeat(H // 16)
    Bc = torch.randn(Bt, T, H, device=dev, generator=g)
    dt = torch.empty(Bt, T, device=dev).exponential_(1.0, generator=g).clamp_(1e-3, 10.0)
    Ab, Bb = ts.zoh_discretize(A_log, Bc, dt)
    dAb = torch.randn(Bt, T, H, device=dev, generator=g)
    dBb = torch.randn(Bt, T, H, device=dev, generator=g)
    a = copy.copy(args)
    a.graph = not args.no_graph
    t_f, clk_f = _timed(a, world, dev, lambda: ts.zoh_discretize(A_log, Bc, dt, out=(Ab, Bb)))
    t_b, clk_b = _timed(a, world, dev, lambda: ts.zoh_discretize_bwd(A_log, Bc, dt, Ab, dAb, dBb))
    n = Bt * T * H
    alg_f = n * 12 + Bt * T * 4 + H * 4
    alg_b = n * 20 + Bt * T * 8 + H * 8
    cfg = {"workload": "zoh_discretize, B%d T%d H%d f32 (config 1's drop-in discretisation)" % (Bt, T, H),
           "global_batch": Bt * world, "seq_len": T, "parallelism": "batch, %d rank(s)" % world,
           "timing": "CUDA-graph replays" if a.graph else "eager launches",
           "l2": "%d MB per step; no flush" % (alg_f // 10**6)}
    out = _line(a, world, METRIC, world * n / t_f, t_f, "f32", cfg, alg_f, "zoh_discretize_kernel<float,1>", None,
                clk_f)
    peak, _ = peaks()
    out["backward"] = {"ms_per_step": t_b * 1e3, "value": world * n / t_b, "unit": UNIT,
                       "kernel": "zoh_discretize_bwd_kernel<1> (+ the dA_log clear)",
                       "algorithmic_bytes_per_launch": alg_b, "achieved_gbs": alg_b / t_b / 1e9,
                       "frac": alg_b / t_b / 1e9 / peak, "clocks": clk_b}
    return out


def run_ours_ring(args, rank, world, local):
    """Streaming ring-buffer ingest + forward fill + step (race-free
    streaming_interp_then_ssm): S=4096 streams, H=1024 features, K=10 (the
    reference's default ring), 128-feature tiles, f32; events cycle through
    16 pre-generated sets, as config 5 does."""
    import triton_ssm_b200 as ts
    dev = torch.device("cuda", local)
    S = args.batch or 4096
    H, K = 1024, 10
    g = torch.Generator(device=dev)
    g.manual_seed(21 + rank)
    ring = ts.StreamingRing(S, H, K, torch.rand(H, device=dev, generator=g) * 0.9,
                            torch.randn(H, device=dev, generator=g), torch.randn(H, device=dev, generator=g),
                            device=dev, block_h=128)
    sets = [dict(v=torch.randn(S, H, device=dev, generator=g),
                 m=(torch.rand(S, H, device=dev, generator=g) < 0.7).float(),
                 tau=torch.rand(S, device=dev, generator=g),
                 C=torch.randn(S, H, device=dev, generator=g)) for _ in range(16)]
    y = torch.empty(S, H, device=dev)
    it = [0]

    def step():
        e = sets[it[0] % 16]
        it[0] += 1
        ring.step(e["v"], e["m"], e["tau"], e["C"], y=y)
    t_step, clocks = _timed(args, world, dev, step)
    # per (stream, feature): event v, m in; ring slot V, M out; h in + out; C in; y out.
    # A tile whose event is observed never reads the ring (with Bernoulli(0.7) masks
    # over 128-feature tiles every tile is observed).
    alg = S * H * 4 * 8 + S * 4 * 2 + H * 4 * 3 + S * 4 * 2
    cfg = {"workload": "ring-buffer streaming step: S%d streams, H%d features, K=%d ring, 128-feature tiles, "
                       "f32, mask Bernoulli(0.7)" % (S, H, K),
           "global_batch": S * world, "seq_len": 1, "parallelism": "streams, %d rank(s)" % world,
           "l2": "state + ring 420 MB per rank, larger than the 126 MB L2"}
    return _line(args, world, METRIC, world * S * H / t_step, t_step, "f32", cfg, alg, "ring_ingest_step_kernel",
                 "ring_ingest_step.md", clocks)


def run_ours_dtproj(args, rank, world, local):
    """Delta-t projection fused into the per-channel ZOH discretisation, H = D*N
    = 1024 as in config 1, dt_rank 64, f32, batch 16 so a step moves more than
    the L2 holds."""
    import triton_ssm_b200 as ts
    dev = torch.device("cuda", local)
    Bt, T, H, R = args.batch or 16, 1024, 1024, 64
    g = torch.Generator(device=dev)
    g.manual_seed(31 + rank)
    dt_raw = torch.randn(Bt, T, R, device=dev, generator=g)
    W = torch.randn(R, H, device=dev, generator=g) / 8.0
    bias = torch.randn(H, device=dev, generator=g) - 3.0
    A_log = torch.log(torch.arange(1, 17, device=dev, dtype=torch.float32)).repeat(64)
    B = torch.randn(Bt, T, H, device=dev, generator=g)
    step = lambda: ts.zoh_discretize_dtproj(A_log, B, dt_raw, W, bias, 1e-3, 1e-1)
    t_step, clocks = _timed(args, world, dev, step)
    n = Bt * T * H
    alg = n * 4 * 3 + Bt * T * R * 4 + R * H * 4 + H * 8
    cfg = {"workload": "delta-t projection (dt_rank %d, softplus, clamp [1e-3, 0.1]) fused into the per-channel "
                       "ZOH discretisation, B%d T%d H%d f32" % (R, Bt, T, H),
           "global_batch": Bt * world, "seq_len": T, "parallelism": "batch, %d rank(s)" % world,
           "l2": "B in + Abar, Bbar out: %d MB per step, larger than the 126 MB L2" % (n * 12 // 1000000)}
    return _line(args, world, METRIC, world * n / t_step, t_step, "f32", cfg, alg, "dtproj_tc_kernel<true> (tcgen05)",
                 "dt_project_discretize.md", clocks)


def _c4_launches(K, world):
    """Kernels of one config-4 step: the scan; with in-device pieces their
    fix-up; with more than one rank the pieces' final state (when K > 1) and
    the slice fix-up (the all-gather is NCCL's)."""
    n = 1 + (1 if K > 1 else 0)
    if world > 1:
        n += (1 if K > 1 else 0) + 1
    return n


def run_ours_c4(args, rank, world, local):
    """Config 4: B4 H32 P64 N128 L=1,048,576 bf16, sequence sharded over the ranks
    (strong scaling): local scan from a zero state, one all-gather of
    (state, decay) per rank, carry fix-up.  The exchange + fix-up time is
    measured on its own from events recorded inside the timed steps."""
    from triton_ssm_b200 import parallel, workloads
    dev = torch.device("cuda", local)
    c = workloads.C4
    Bt, H, P, N = c["Bt"], c["H"], c["P"], c["N"]
    L = args.seq_len or c["L"]
    a, b = parallel.shard_range(L // (1 << 14), rank, world)
    L0, Ls = a * (1 << 14), (b - a) * (1 << 14)
    inp = workloads.ssd_inputs_slice(Bt, L0, Ls, H, P, N, dev, seed=4)
    y = torch.empty_like(inp["x"])
    step = lambda marks=None: parallel.ssd_sequence_parallel(inp["x"], inp["dt"], inp["A_log"], inp["B"], inp["C"],
                                                              inp["D"], y=y, marks=marks)
    stream = torch.cuda.current_stream(dev)
    t_step, clocks = _timed(args, world, dev, step)
    # a separate pass with events around each step splits scan / exchange + fix-up
    n_split = max(3, min(args.steps, 10))
    starts, ends, marks = [], [], []
    torch.cuda.synchronize()
    barrier(world)
    for _ in range(n_split):
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step(marks)
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record(stream)
        starts.append(e0)
        ends.append(e1)
    torch.cuda.synchronize()
    scan_ms = statistics.median(s.elapsed_time(m) for s, m in zip(starts, marks))
    xfix_ms = statistics.median(m.elapsed_time(e) for m, e in zip(marks, ends))
    xfix_min_ms = min_over_ranks(xfix_ms, world)
    scan_ms = max_over_ranks(scan_ms, world)
    xfix_ms = max_over_ranks(xfix_ms, world)
    upd = Bt * L * H * P * N
    alg = workloads.ssd_bytes(Bt, L, H, P, N)
    K = parallel.ssd_local_pieces(Bt, H, Ls, torch.cuda.get_device_properties(dev).multi_processor_count)
    cfg = {"workload": "config4: sequence-parallel multi-head scan B%d H%d P%d N%d L=%d bf16, A_h=-(1+h%%16), "
                       "L sharded over %d rank(s) with one all-gather of slice carries" % (Bt, H, P, N, L, world),
           "global_batch": Bt, "seq_len": L, "parallelism": "sequence (L) x %d" % world,
           "slice_tokens_per_rank": Ls, "in_device_pieces": K,
           "nvlink_bytes_per_rank": Bt * H * P * N * 4 + Bt * H * 4,
           "l2": "%d GB of inputs and outputs per rank per step (> the 126 MB L2)" % (alg // world // 10**9)}
    out = _line(args, world, METRIC, upd / t_step, t_step, "bf16", cfg, alg // world,
                "ssd_chunk_scan_kernel<128,false> + ssd_carry_fixup_kernel<128>",
                "ssd_chunk_scan_c4.md" if L == c["L"] else None, clocks,
                launches=_c4_launches(K, world) * args.steps)
    if out["roofline"]["traffic"] is not None and world > 1:
        out["roofline"]["traffic"] //= world
        out["roofline"]["traffic_note"] = "full-size 1-GPU capture divided by the rank count"
    out["scaling"] = "strong"
    out["roofline"]["note"] = "algorithmic bytes per rank (1/world of the whole sequence)"
    out["split_ms"] = {"local_scan": scan_ms, "exchange_and_fixup": xfix_ms,
                       "exchange_and_fixup_frac": xfix_ms / max(1e-9, scan_ms + xfix_ms),
                       "exchange_and_fixup_min_rank": xfix_min_ms,
                       "exchange_and_fixup_min_rank_frac": xfix_min_ms / max(1e-9, scan_ms + xfix_ms),
                       "how": "median over %d steps of CUDA events before the step, after the local scan, after "
                              "the fix-up; max over ranks (which includes a fast rank waiting in the all-gather for "
                              "the slowest rank's local scan) and min over ranks (about the exchange and fix-up "
                              "alone)" % n_split}
    del inp, y
    return out


def run_ours_c4_bh(args, rank, world, local):
    """Config 4 sharded by batch x head instead of by sequence, for comparison:
    rank r scans heads [r H/world, (r+1) H/world) of every batch over the whole
    L, each sequence cut into in-device pieces so that the rank's few streams
    still fill its SMs; no collective."""
    import triton_ssm_b200 as ts
    from triton_ssm_b200 import parallel, workloads
    dev = torch.device("cuda", local)
    c = workloads.C4
    Bt, H, P, N = c["Bt"], c["H"], c["P"], c["N"]
    L = args.seq_len or c["L"]
    h0, h1 = parallel.shard_range(H, rank, world)
    Hl = h1 - h0
    inp = workloads.ssd_inputs_slice(Bt, 0, L, Hl, P, N, dev, seed=40 + rank)
    inp["A_log"] = torch.log(1.0 + ((h0 + torch.arange(Hl, device=dev)) % 16).float())   # A_h = -(1 + h mod 16)
    K = parallel.ssd_local_pieces(Bt, Hl, L, torch.cuda.get_device_properties(dev).multi_processor_count)
    y = torch.empty_like(inp["x"])
    step = lambda: ts.multihead_ssm(inp["x"], inp["A_log"], inp["B"], inp["C"], inp["dt"], inp["D"], y=y, pieces=K)
    t_step, clocks = _timed(args, world, dev, step)
    upd = Bt * L * H * P * N
    alg = workloads.ssd_bytes(Bt, L, H, P, N)
    cfg = {"workload": "config4 sharded by batch x head: B%d H%d P%d N%d L=%d bf16, %d head(s) of every batch per "
                       "rank over the whole sequence, %d in-device pieces, no collective" % (Bt, H, P, N, L, Hl, K),
           "global_batch": Bt, "seq_len": L, "parallelism": "batch x head over %d rank(s)" % world,
           "heads_per_rank": Hl, "in_device_pieces": K}
    out = _line(args, world, METRIC, upd / t_step, t_step, "bf16", cfg, alg // world,
                "ssd_chunk_scan_kernel<128,false> + ssd_carry_fixup_kernel<128>", None, clocks,
                launches=(1 + (K > 1)) * args.steps)
    out["scaling"] = "strong"
    out["roofline"]["note"] = "algorithmic bytes per rank (1/world of the whole problem)"
    del inp, y
    return out


def run_ours_c2(args, rank, world, local):
    import triton_ssm_b200 as ts
    from triton_ssm_b200 import workloads
    ts.load_library()
    dev = torch.device("cuda", local)
    c = workloads.C2
    Bt, L, H, P, N = args.batch or c["Bt"], c["L"], c["H"], c["P"], c["N"]
    inp = workloads.ssd_inputs(Bt, L, H, P, N, dev, seed=1234 + rank)
    y = torch.empty_like(inp["x"])
    step = lambda: ts.multihead_ssm(inp["x"], inp["A_log"], inp["B"], inp["C"], inp["dt"], inp["D"], y=y)
    t_step, clocks = _timed(args, world, dev, step)
    upd = workloads.ssd_updates(Bt, L, H, P, N)
    value = world * upd / t_step
    alg_bytes = workloads.ssd_bytes(Bt, L, H, P, N)

    # ---- end to end through the public host-buffer API (pinned host memory)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e_c2(inp, y, Bt, L, H, P, N, dev, args, world, upd, t_step)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        r, thr, sample = cpu_ssd_rate(Bt, H, P, N, 512, args.cpu_seconds)
        cpu = {"value": r, "unit": UNIT, "cores": thr, "kind": "port", "sample": sample}
    cfg = {"workload": "config2: multi-head chunked scan (SSD state) B%d H8 P64 N64 L8192, "
                       "chunk 256 (kernel tile 64), Euler B, bf16 in / f32 state" % Bt,
           "global_batch": Bt * world, "seq_len": L, "heads": H, "head_dim": P, "d_state": N,
           "parallelism": "batch x head, %d independent rank(s)" % world,
           "l2": "inputs (%d MB/step) larger than the 126 MB L2; no flush" % (alg_bytes // 2**20)}
    return _line(args, world, METRIC, value, t_step, "bf16", cfg, alg_bytes, "ssd_chunk_scan_kernel<64,false>",
                 "ssd_chunk_scan_c2.md", clocks, cpu=cpu, e2e=e2e)


def run_e2e_c2(inp, y, Bt, L, H, P, N, dev, args, world, upd, t_kernel):
    from triton_ssm_b200.host import SSDHostPipeline, bind_host_to_gpu, pinned_copy_gbs
    e2e_steps = max(3, min(args.steps, 20))
    # pinned buffers on the GPU's NUMA node, then the host link measured with
    # every rank copying at once (the bound the host-buffer path runs against)
    affinity = os.sched_getaffinity(0)
    numa = bind_host_to_gpu(dev)
    barrier(world)
    h2d_gbs, d2h_gbs = pinned_copy_gbs(dev)
    # the slowest rank's link
    h2d_gbs = 1.0 / max_over_ranks(1.0 / h2d_gbs, world)
    d2h_gbs = 1.0 / max_over_ranks(1.0 / d2h_gbs, world)
    barrier(world)
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
    os.sched_setaffinity(0, affinity)   # the CPU-baseline leg after this uses every allowed core again
    # spot-check the host result against the device result
    if not torch.equal(y_h.to(dev), y):
        raise RuntimeError("host-pipeline output differs from the device run")
    h2d_ms = pipe.h2d_bytes() / (h2d_gbs * 1e9) * 1e3
    return {"value": world * upd / e2e_t, "unit": UNIT, "h2d_bytes_per_step": pipe.h2d_bytes(),
            "d2h_bytes_per_step": pipe.d2h_bytes(), "ms_per_step": e2e_t * 1e3, "steps": e2e_steps,
            "gpu_launches": len(pipe.slices) * e2e_steps,
            "path": "triton_ssm_b200.host.SSDHostPipeline (pinned host buffers, 8 batch slices)",
            "host_link": {"h2d_gbs": round(h2d_gbs, 2), "d2h_gbs": round(d2h_gbs, 2),
                          "numa_node": numa["numa_node"] if numa else None,
                          "bound_cpus": numa["cpus"] if numa else None,
                          "binding": numa["source"] if numa else "none (one NUMA node, or the GPU's CPUs are all allowed ones)",
                          "how": "256 MiB pinned copies timed with CUDA events, all %d rank(s) at once" % world},
            "limit": "host->device copies: %.2f ms of the %.2f ms step at the slowest rank's measured %.1f GB/s; "
                     "the scan kernel is %.3f ms" % (h2d_ms, e2e_t * 1e3, h2d_gbs, t_kernel * 1e3)}


SUB_KEYS = ("metric", "value", "unit", "ms_per_step", "steps", "warmup", "scaling", "dtype", "config", "roofline",
            "gpu_launches", "clocks", "steps_per_sec", "p50_step_ms", "p99_step_ms", "split_ms", "n_gpus")


def run_sub_configs(args, rank, world, local):
    """The other benchmark configs, each timed like the headline (warm-up, a
    second of load, exactly `steps` CUDA-event-timed steps, clocks sampled),
    reported as sub-records of the one JSON line.  Config 4 is the sequence-
    sharded scan over all ranks (its one collective), and, with more than one
    rank, config 4 sharded by batch x head for comparison ("c4_bh"); configs
    1, 3 and 5 run on a single GPU (only when world == 1)."""
    import copy
    out = {}
    names = [c.strip() for c in args.configs.split(",") if c.strip()]
    runners = {"c1": run_ours_c1, "c3": run_ours_c3, "c4": run_ours_c4, "c5": run_ours_c5,
               "c4_bh": run_ours_c4_bh}
    if world > 1 and "c4" in names and "c4_bh" not in names:
        names.insert(names.index("c4") + 1, "c4_bh")   # the batch x head sharding of config 4, for comparison
    for name in names:
        if name not in runners:
            raise SystemExit("unknown sub-config %r" % name)
        if name not in ("c4", "c4_bh") and world > 1:
            continue
        a = copy.copy(args)
        a.batch = None
        a.graph = name == "c1" and not args.no_graph
        torch.cuda.empty_cache()
        rec = runners[name](a, rank, world, local)
        out[name] = {k: rec[k] for k in SUB_KEYS if k in rec}
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return out


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
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c4", "c5", "c1bwd", "ring", "dtproj", "disc"], default="c2",
                    help="workload (default c2, the headline; the others are for measurement notes)")
    ap.add_argument("--c1-mode", choices=["pair", "fused", "pool"], default="pair")
    ap.add_argument("--graph", action="store_true", help="time CUDA-graph replays of the step")
    ap.add_argument("--no-graph", action="store_true",
                    help="config 1: time the eager per-op launches instead of graph replays")
    ap.add_argument("--seq-len", type=int, default=None, help="config 4: override L (multiple of 16384)")
    ap.add_argument("--configs", default="c4,c1,c3,c5",
                    help="with the default config 2 line: the other configs timed in the same process and reported "
                         "under 'configs' (c4 on every rank, sequence-sharded; c1/c3/c5 on one GPU only); "
                         "'none' to skip")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    # Config 1 (forward and backward) is two ~10-30 us kernels: eager Python dispatch of the two operators
    # costs more than they run, so its steps are captured once and replayed as a
    # CUDA graph (the same kernels and bytes; the host launch path is what goes).
    if args.config in ("c1", "c1bwd") and not args.no_graph:
        args.graph = True
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
        runner = {"c1": run_ours_c1, "c2": run_ours_c2, "c3": run_ours_c3, "c4": run_ours_c4,
                  "c5": run_ours_c5, "c1bwd": run_ours_c1bwd, "ring": run_ours_ring,
                  "dtproj": run_ours_dtproj, "disc": run_ours_disc}[args.config]
        out = runner(args, rank, world, local)
        if args.config == "c2" and args.configs != "none":
            out["configs"] = run_sub_configs(args, rank, world, local)
        if rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
