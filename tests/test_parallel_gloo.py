"""Multi-process (gloo, CPU) tests of the sequence-parallel orchestration and of
failure handling between ranks.  The CUDA operators are replaced by the CPU
oracle, so these run without a GPU; the kernels themselves are checked on the
GPU in tests/test_gpu_parallel.py."""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(seed=0, Bt=2, L=96, H=2, P=4, N=3):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(Bt, L, H * P, generator=g)
    dt = torch.exp(torch.empty(Bt, L, H).uniform_(-4.0, 0.0, generator=g))
    A_log = torch.empty(H).uniform_(-0.7, 2.7, generator=g)
    B = torch.randn(Bt, L, H, N, generator=g) / N ** 0.5
    C = torch.randn(Bt, L, H, N, generator=g) / N ** 0.5
    D = torch.randn(H * P, generator=g)
    return x, dt, A_log, B, C, D


def _worker_sp(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    import datetime

    import torch.distributed as dist

    import oracle
    from triton_ssm_b200 import parallel
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    x, dt, A_log, B, C, D = _inputs()
    L = x.shape[1]
    a, b = parallel.shard_range(L, rank, world)
    y = parallel.ssd_sequence_parallel(
        x[:, a:b].contiguous(), dt[:, a:b].contiguous(), A_log, B[:, a:b].contiguous(), C[:, a:b].contiguous(), D,
        local_scan=lambda *t: oracle.ssd_slice_scan(*t), fixup=oracle.ssd_carry_fixup)
    torch.save(y, os.path.join(out_dir, "y%d.pt" % rank))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sequence_parallel_matches_single_rank(tmp_path, world):
    import oracle
    mp.spawn(_worker_sp, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    y = torch.cat([torch.load(os.path.join(tmp_path, "y%d.pt" % r)) for r in range(world)], dim=1)
    x, dt, A_log, B, C, D = _inputs()
    ref, _ = oracle.ssd_scan(x, dt, A_log, B, C, D)
    assert ((y - ref).abs().max() / ref.abs().max()).item() < 1e-5


def test_shard_range_covers_exactly():
    from triton_ssm_b200 import parallel
    for n in (0, 1, 7, 128, 1000):
        for w in (1, 2, 3, 8):
            parts = [parallel.shard_range(n, r, w) for r in range(w)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(w - 1))
            assert max(p[1] - p[0] for p in parts) - min(p[1] - p[0] for p in parts) <= 1


def _worker_fail(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    import datetime
    import time

    import torch.distributed as dist
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        # a rank that dies between steps, with nothing in flight
        os._exit(3)
    t0 = time.time()
    try:
        buf = [torch.zeros(4) for _ in range(world)]
        dist.all_gather(buf, torch.ones(4))
        status = "no-error"
    except Exception as e:   # the survivor must get an error, not hang
        status = "error:" + type(e).__name__
    with open(os.path.join(out_dir, "status%d.txt" % rank), "w") as f:
        f.write("%s %.1f" % (status, time.time() - t0))
    os._exit(0)


def test_dead_rank_surfaces_as_error_not_hang(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker_fail, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert not p.is_alive(), "a rank hung"
    status, secs = open(os.path.join(tmp_path, "status0.txt")).read().split()
    assert status.startswith("error"), status
    assert float(secs) < 60
